"""GPU parity: the CUDA engine (through the C ABI) against the CPU oracle.

The engine and the oracle implement the same arithmetic op by op, so the bar
is bit-identity: token ids equal, logits equal as float32 bit patterns, cross
K/V equal as f16 bit patterns. The reference's own GPU test is
fused_gpu_decoding_matches_the_reference_path (crates/malaga-core/tests/
pipeline.rs:108-124: tiny model, f32 and q8_0 presets, 6 sentences, second run
replays the cached graphs); these tests cover that and the quantized presets
at NLLB widths.
"""
import numpy as np
import pytest

import oracle
from malaga_b200 import Engine, GenOptions, MgbError, Translator
from malaga_b200 import convert as C
from malaga_b200 import models

pytestmark = pytest.mark.gpu

TINY_SRC, TINY_TGT = 254, 256


def tiny_sentences():
    # pipeline.rs:132-134: sentence(3 + 4i, i) for i in 0..6, wrapped [src] ... [eos]
    return [[TINY_SRC] + C.tiny_sentence(3 + 4 * i, i) + [2] for i in range(6)]


def mid_sentences(vocab, n=5, seed=3):
    return models.random_sources(n, 3, 20, vocab, seed, src_tag=vocab - 1)


@pytest.mark.parametrize("preset", ["f32", "q8_0", "q4_k_m"])
def test_tiny_greedy_tokens_and_logits_bit_exact(gpu, model, preset):
    path = model("tiny", preset)
    src = tiny_sentences()
    orc = oracle.Oracle(path)
    want_ids, want_logits = orc.greedy(src, TINY_TGT, 12, logits=True)
    eng = Engine(path)
    batch = eng.encode(src)
    got_ids, got_logits = eng.greedy_logits(batch, TINY_TGT, 12)
    np.testing.assert_array_equal(got_ids, want_ids)
    # finished rows emit pad but still compute logits; compare every row
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32)), \
        f"max |diff| {np.abs(got_logits - want_logits).max()}"


@pytest.mark.parametrize("name,preset", [("mid", "q4_k_m"), ("mid", "q8_0"), ("wide", "q4_k_m"), ("wide", "q8_0")])
def test_quantized_widths_bit_exact(gpu, model, name, preset):
    path = model(name, preset)
    V = models.config_of(name).vocab_size
    src = mid_sentences(V)
    tgt = V - 2
    orc = oracle.Oracle(path)
    want_ids, want_logits = orc.greedy(src, tgt, 6, force=True, logits=True)
    eng = Engine(path)
    batch = eng.encode(src)
    got_ids, got_logits = eng.greedy_logits(batch, tgt, 6, force=True)
    np.testing.assert_array_equal(got_ids, want_ids)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32)), \
        f"max |diff| {np.abs(got_logits - want_logits).max()}"
    # north_star tolerance, stated for the record (bit-identity is stronger)
    assert np.abs(got_logits - want_logits).max() <= 2e-2


@pytest.mark.parametrize("name,preset", [("tiny", "q8_0"), ("mid", "q4_k_m"), ("wide", "q8_0")])
def test_encoder_cross_kv_bit_exact(gpu, model, name, preset):
    path = model(name, preset)
    V = models.config_of(name).vocab_size
    src = tiny_sentences() if name == "tiny" else mid_sentences(V)
    orc = oracle.Oracle(path)
    enc = orc.encode(src)
    eng = Engine(path)
    batch = eng.encode(src)
    for layer in range(models.config_of(name).decoder_layers):
        for which in (0, 1):
            want = orc.cross(enc, layer, which).astype(np.float16)
            got = eng.cross(batch, layer, which)
            assert np.array_equal(got.view(np.uint16), want.view(np.uint16)), (layer, which)


@pytest.mark.parametrize("preset", ["f32", "q8_0"])
def test_graph_replay_matches_eager_and_oracle(gpu, model, preset):
    """pipeline.rs:108-124: fused == reference, and a second run replays the graph."""
    path = model("tiny", preset)
    src = tiny_sentences()
    orc = oracle.Oracle(path)
    want = orc.greedy(src, TINY_TGT, 20)
    eng = Engine(path)
    t = Translator(eng)
    opts = GenOptions(max_new_tokens=20)
    first = t.generate(src, TINY_TGT, opts)
    launches = eng.kernel_launches
    second = t.generate(src, TINY_TGT, opts)
    assert eng.kernel_launches > launches
    eager = Translator(Engine(path, use_graphs=False)).generate(src, TINY_TGT, opts)
    expect = [oracle.strip_eos(r, 2) for r in want]
    assert first == expect
    assert second == expect
    assert eager == expect


def test_batching_does_not_change_outputs(gpu, model):
    """pipeline.rs:45-57 (batch == single) on the f32 preset, as the reference
    tests it: quantized presets depend on the batch size in the reference
    (docs/performance.md:51-54) and here alike."""
    path = model("tiny", "f32")
    src = tiny_sentences()
    t = Translator(Engine(path))
    opts = GenOptions(max_new_tokens=10, force_steps=True)
    batched = t.generate(src, TINY_TGT, opts)
    for s, row in zip(src, batched):
        assert t.generate([s], TINY_TGT, opts)[0] == row


def test_idle_rows_sync_every_and_eos(gpu, model):
    """Batch 5 runs in a bucket of 8 idle-padded rows; the early exit every
    sync_every steps and the eos truncation match the oracle."""
    path = model("tiny", "q8_0")
    src = tiny_sentences()[:5]
    orc = oracle.Oracle(path)
    want = [oracle.strip_eos(r, 2) for r in orc.greedy(src, TINY_TGT, 30)]
    eng = Engine(path)
    for sync_every in (1, 3, 4):
        out, lens = eng.greedy(eng.encode(src), TINY_TGT, 30, sync_every=sync_every)
        assert [list(map(int, out[i, : lens[i]])) for i in range(5)] == want


def test_translate_batch_sorted_order_and_budget(gpu, model):
    """translate_batch: length-sorted chunks of max_batch, input order kept,
    per-sentence budget 2*len+16 (translator.rs:136-207)."""
    path = model("tiny", "q8_0")
    src = tiny_sentences()
    t = Translator(Engine(path))
    out = t.translate_batch(src, TINY_TGT, GenOptions(max_batch=2))
    orc = oracle.Oracle(path)
    for s, row in zip(src, out):
        budget = min(2 * len(s) + 16, 64)
        want = oracle.strip_eos(orc.greedy([s], TINY_TGT, budget)[0], 2)[:budget]
        assert row == want


def test_injected_oom_is_reported_and_recovered(gpu, model):
    """Allocation failure -> MGB_ERR_OOM with the reference's OUT_OF_MEMORY text;
    the context stays usable (graph.rs:214-222, translator.rs:150-158)."""
    path = model("tiny", "q8_0")
    src = tiny_sentences()
    eng = Engine(path, fail_alloc_after=1)  # the batch buffer (after the encoder workspace)
    with pytest.raises(MgbError) as e:
        eng.encode(src)
    assert e.value.is_oom
    # later allocations succeed: the same context decodes correctly
    want = [oracle.strip_eos(r, 2) for r in oracle.Oracle(path).greedy(src, TINY_TGT, 10)]
    got = Translator(eng).generate(src, TINY_TGT, GenOptions(max_new_tokens=10))
    assert got == want


def test_batch_buffers_are_pooled_and_outlive_close(gpu, model):
    """Freed batches' device buffers are reused by later encodes (a larger one
    for a smaller batch too) with unchanged results; a batch freed after its
    context was closed releases its own buffer."""
    path = model("tiny", "q8_0")
    src = tiny_sentences()
    orc = oracle.Oracle(path)
    eng = Engine(path)
    for batch in (src, src[:2], src, src[:1]):
        want = [oracle.strip_eos(r, 2) for r in orc.greedy(batch, TINY_TGT, 8)]
        b = eng.encode(batch)
        out, lens = eng.greedy(b, TINY_TGT, 8)
        b.free()
        assert [[int(x) for x in out[i, : lens[i]]] for i in range(len(batch))] == want
    b = eng.encode(src)
    eng.close()
    b.free()


def test_invalid_arguments_fail_cleanly(gpu, model):
    eng = Engine(model("tiny", "q8_0"))
    with pytest.raises(MgbError):
        eng.encode([[300, 2]])  # id >= vocab
    b = eng.encode(tiny_sentences()[:1])
    with pytest.raises(MgbError):
        eng.greedy(b, 999, 4)  # target id >= vocab
    with pytest.raises(MgbError):
        eng.greedy(b, TINY_TGT, 0)


@pytest.mark.slow
def test_600m_q4_k_m_b1_config1_all_steps_bit_exact(gpu, model):
    """Config 1 at full size (NLLB-600M q4_k_m, 34-token source, batch 1): all
    32 forced steps, tokens and logits, against the oracle."""
    path = model("600m", "q4_k_m")
    w = models.workload("c1")
    orc = oracle.Oracle(path)
    want_ids, want_logits = orc.greedy(w.sources, models.TGT_TAG, w.steps, force=True, logits=True)
    eng = Engine(path)
    got_ids, got_logits = eng.greedy_logits(eng.encode(w.sources), models.TGT_TAG, w.steps, force=True)
    np.testing.assert_array_equal(got_ids, want_ids)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))


@pytest.mark.slow
def test_600m_q8_0_b64_config2_prefix_bit_exact(gpu, model):
    """Config 2 at full size (NLLB-600M q8_0, 64 sentences of 8-64 tokens): the
    encoder and 3 forced steps on the tensor-core path, against the oracle."""
    w = models.workload("c2")
    path = model(w.model, w.preset, w.seed)
    orc = oracle.Oracle(path)
    want_ids, want_logits = orc.greedy(w.sources, models.TGT_TAG, 3, force=True, logits=True)
    eng = Engine(path)
    got_ids, got_logits = eng.greedy_logits(eng.encode(w.sources), models.TGT_TAG, 3, force=True)
    np.testing.assert_array_equal(got_ids, want_ids)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))


@pytest.mark.parametrize("preset", ["q4_k_m", "q8_0"])
@pytest.mark.parametrize("n", [3, 20])
def test_3_3b_layer_shapes_bit_exact(gpu, model, preset, n):
    """The 3.3B layer shapes (d_model 2048, 16 heads of 128, FFN 8192; 2+2 layers,
    16k vocabulary): 3 rows on the small-batch kernels, 20 rows (a 32-row bucket)
    on the tensor cores, encoder included; tokens and logits bit-exact."""
    path = model("3.3b-lite", preset)
    V = models.config_of("3.3b-lite").vocab_size
    src = models.random_sources(n, 3, 14, V, 31, src_tag=V - 1)
    want_ids, want_logits = oracle.Oracle(path).greedy(src, V - 2, 3, force=True, logits=True)
    eng = Engine(path)
    got_ids, got_logits = eng.greedy_logits(eng.encode(src), V - 2, 3, force=True)
    np.testing.assert_array_equal(got_ids, want_ids)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32)), \
        f"max |diff| {np.abs(got_logits - want_logits).max()}"


def test_bounded_wait_that_runs_out_is_reported(gpu, model, monkeypatch):
    """A bounded mbarrier wait that runs out: the test hook withholds one weight
    copy of the small-batch kernel's first CTA and shortens the limit to 20 ms;
    the kernel records the error word and returns (no hang, no fault), the call
    fails with MGB_ERR_CUDA, and a context opened afterwards decodes correctly."""
    from malaga_b200 import _lib

    path = model("tiny", "q8_0")
    src = tiny_sentences()[:1]  # 1 sentence: the encoder's matmuls run the small-batch kernel
    monkeypatch.setenv("MGB_TEST_WAIT_NS", "20000000")
    monkeypatch.setenv("MGB_TEST_WITHHOLD_CHUNK", "0")
    eng = Engine(path)
    with pytest.raises(MgbError) as e:
        eng.encode(src)
    assert e.value.code == _lib.MGB_ERR_CUDA
    assert "ran out of time" in str(e.value)
    eng.close()
    monkeypatch.delenv("MGB_TEST_WAIT_NS")
    monkeypatch.delenv("MGB_TEST_WITHHOLD_CHUNK")
    want = [oracle.strip_eos(r, 2) for r in oracle.Oracle(path).greedy(src, TINY_TGT, 8)]
    assert Translator(Engine(path)).generate(src, TINY_TGT, GenOptions(max_new_tokens=8)) == want


@pytest.mark.parametrize("chunk", [0, 3])
def test_bounded_wait_in_step_kernel_is_reported(gpu, model, monkeypatch, chunk):
    """The persistent step kernel's failure path: the test hook withholds one
    weight copy of CTA 0 (the first chunk, or one of a later phase) and shortens
    every wait to 20 ms; the warps that wait for it give up and raise the abort
    flag, the other CTAs leave at their next grid barrier, every CTA waits for its
    own copies in flight, and the call fails with MGB_ERR_CUDA instead of hanging.
    A context opened afterwards decodes correctly."""
    from malaga_b200 import _lib

    path = model("mid", "q8_0")
    V = models.config_of("mid").vocab_size
    src = mid_sentences(V, n=1, seed=21)
    monkeypatch.setenv("MGB_STEP_KERNEL", "1")
    monkeypatch.setenv("MGB_TEST_WAIT_NS", "20000000")
    monkeypatch.setenv("MGB_TEST_WITHHOLD_STEP", str(chunk))
    eng = Engine(path)
    batch = eng.encode(src)
    with pytest.raises(MgbError) as e:
        eng.greedy_logits(batch, V - 2, 2, force=True)
    assert e.value.code == _lib.MGB_ERR_CUDA
    assert "ran out of time" in str(e.value)
    eng.close()
    monkeypatch.delenv("MGB_TEST_WAIT_NS")
    monkeypatch.delenv("MGB_TEST_WITHHOLD_STEP")
    want_ids, _ = oracle.Oracle(path).greedy(src, V - 2, 4, force=True, logits=True)
    eng = Engine(path)
    got, _ = eng.greedy(eng.encode(src), V - 2, 4, force=True)
    np.testing.assert_array_equal(got, want_ids)


@pytest.mark.parametrize("name,preset,b,ffn_q8", [("mid", "q4_k_m", 64, "0"), ("mid", "q8_0", 24, "0"),
                                                  ("wide", "q8_0", 64, "0"), ("wide", "q4_k_m", 40, "0"),
                                                  ("wide", "q4_k_m", 40, "1"), ("mid", "q8_0", 24, "1"),
                                                  ("mid", "q4_k_m", 128, "0")])
def test_tensor_core_batches_bit_exact(gpu, model, name, preset, b, ffn_q8, monkeypatch):
    """Batches of 16+ rows run the tcgen05 matmuls (and the encoder always does for
    quantized weights): tokens and logits equal the oracle's bit for bit. ffn_q8 1:
    the FFN-up epilogue quantizes the down matmul's activations itself."""
    monkeypatch.setenv("MGB_FFN_Q8", ffn_q8)
    path = model(name, preset)
    V = models.config_of(name).vocab_size
    src = models.random_sources(b, 2, 10, V, 11, src_tag=V - 1)
    orc = oracle.Oracle(path)
    want_ids, want_logits = orc.greedy(src, V - 2, 3, force=True, logits=True)
    eng = Engine(path)
    got_ids, got_logits = eng.greedy_logits(eng.encode(src), V - 2, 3, force=True)
    np.testing.assert_array_equal(got_ids, want_ids)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32)), \
        f"max |diff| {np.abs(got_logits - want_logits).max()}"


@pytest.mark.parametrize("mode", ["two_contexts", "four_contexts", "64"])
@pytest.mark.parametrize("name,preset,b", [("mid", "q4_k_m", 64), ("wide", "q4_k_m", 40)])
def test_tensor_core_tile_floors_bit_exact(gpu, model, name, preset, b, mode, monkeypatch):
    """With several contexts open on the device the tensor-core matmuls use wider
    token tiles (16 tokens at least for two contexts, 32 from four, 64 with
    MGB_TC_MIN_NT=64); the tiles change which CTA forms an output, not its
    arithmetic: tokens and logits equal the oracle's bit for bit."""
    if mode == "64":
        monkeypatch.setenv("MGB_TC_MIN_NT", mode)
    path = model(name, preset)
    V = models.config_of(name).vocab_size
    src = models.random_sources(b, 2, 10, V, 11, src_tag=V - 1)
    want_ids, want_logits = oracle.Oracle(path).greedy(src, V - 2, 3, force=True, logits=True)
    eng = Engine(path)
    others = [Engine(path) for _ in range({"two_contexts": 1, "four_contexts": 3}.get(mode, 0))]
    got_ids, got_logits = eng.greedy_logits(eng.encode(src), V - 2, 3, force=True)
    for o in others:
        o.close()
    np.testing.assert_array_equal(got_ids, want_ids)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32)), \
        f"max |diff| {np.abs(got_logits - want_logits).max()}"


@pytest.mark.parametrize("name,preset,n,k", [("tiny", "q8_0", 6, 3), ("tiny", "f32", 4, 2), ("mid", "q4_k_m", 4, 4),
                                             ("mid", "q8_0", 3, 5), ("mid", "q4_k_m", 1, 3), ("mid", "q8_0", 2, 2)])
def test_beam_search_matches_oracle(gpu, model, name, preset, n, k):
    """Beam search (translator.rs:250-358) on the reference's generic decode: f32
    self / cross K/V, the [</s>, tgt] prefill with the row class of a 2-token
    call, device log_softmax + top-k, host merge; the hypotheses equal the
    oracle's (mid q4_k_m 4x4: 16 rows run the tcgen05 step; 1x3: 3 rows on the
    small kernels with a 6-row (2-warp) prefill; 2x2: 4 rows, 8-row prefill)."""
    path = model(name, preset)
    if name == "tiny":
        src, tgt = tiny_sentences()[:n], TINY_TGT
    else:
        V = models.config_of(name).vocab_size
        src, tgt = mid_sentences(V, n=n, seed=9), V - 2
    want = oracle.Oracle(path).beam(src, tgt, k, 12)
    eng = Engine(path)
    out, lens = eng.beam(eng.encode(src), tgt, k, 12)
    got = [[int(t) for t in out[i, : lens[i]]] for i in range(len(src))]
    assert got == [[int(t) for t in r] for r in want]


@pytest.mark.slow
def test_beam_config3_row_shape_full_vocabulary(gpu, model):
    """Config 3's shape: beam 4 over 16 sources of 48 tokens (64 beam rows on the
    tensor cores, a 128-row prefill), d_model 1024, FFN 8192 and the full 256206
    vocabulary (2+2 layers): the hypotheses equal the oracle's."""
    path = model("1.3b-lite", "q4_k_m", 2)
    V = models.config_of("1.3b-lite").vocab_size
    src = models.random_sources(16, 46, 46, V, 2, fixed_len=46)  # tag + 46 ids + </s> = 48
    want = oracle.Oracle(path).beam(src, models.TGT_TAG, 4, 8)
    eng = Engine(path)
    out, lens = eng.beam(eng.encode(src), models.TGT_TAG, 4, 8)
    got = [[int(t) for t in out[i, : lens[i]]] for i in range(len(src))]
    assert got == [[int(t) for t in r] for r in want]


def _topk_rows(rng, V):
    """Adversarial logits rows of width V (finite or partly -inf)."""
    rows = [rng.standard_normal(V).astype(np.float32) * 4.0,                  # spread, one clear leader
            rng.integers(-3, 4, V).astype(np.float32),                         # massive ties
            np.full(V, 1.5, np.float32),                                       # all equal
            (rng.standard_normal(V) * 100.0).astype(np.float32)]              # most exps underflow
    r = rng.standard_normal(V).astype(np.float32)
    r[rng.random(V) < 0.9] = -np.inf                                           # mostly -inf
    r[0] = 0.25
    rows.append(r)
    r = np.full(V, -np.inf, np.float32)
    r[V - 1] = -7.0                                                            # one finite value, last index
    rows.append(r)
    return np.stack(rows)


@pytest.mark.parametrize("V", [1, 5, 31, 33, 4096, 4097, 12289, 256206, 600000])
@pytest.mark.parametrize("k", [1, 4, 8])
def test_log_softmax_topk_kernel_bit_exact(gpu, model, V, k):
    """The beam step's device half (log_softmax + top-k, translator.rs:343-358)
    on caller logits: values as f32 bit patterns and indices equal the oracle's
    on ties, all-equal rows, underflowing exponentials, -inf runs, rows shorter
    than k (padded with (-inf, 0)), rows that start off a 16-byte boundary (odd
    rows of odd V), one to 147 streamed chunks and rows too long to keep chunk
    maxima (600000 > 128 chunks: every chunk scanned)."""
    rng = np.random.default_rng(V * 10 + k)
    x = _topk_rows(rng, V)
    want_v, want_i = oracle.log_softmax_topk(x, k)
    eng = Engine(model("tiny", "q8_0"))
    got_v, got_i = eng.log_softmax_topk(x, k)
    np.testing.assert_array_equal(got_i, want_i)
    assert np.array_equal(got_v.view(np.uint32), want_v.view(np.uint32)), (got_v, want_v)


@pytest.mark.parametrize("position", [0, 70, 130])
def test_topk_bounded_wait_that_runs_out_is_reported(gpu, model, position, monkeypatch):
    """The top-k kernel's bounded waits: the test hook withholds the bulk copy at
    one ring position of row 0 (positions 0-64: the max pass of a 65-chunk row,
    65-129: the exponential pass, 130: the first chunk of the top-k pass) and shortens the limit to 20 ms; the kernel sets the
    error word and returns, the call fails with MGB_ERR_CUDA, and a context
    opened afterwards gives the oracle's result."""
    from malaga_b200 import _lib

    rng = np.random.default_rng(position)
    x = rng.standard_normal((3, 4096 * 64 + 5)).astype(np.float32)  # 65 chunks per row
    x[0, 4096 * 64 + 2] = 9.0  # row 0's winner in its last chunk: the top-k pass fetches it
    monkeypatch.setenv("MGB_TEST_WAIT_NS", "20000000")
    monkeypatch.setenv("MGB_TEST_WITHHOLD_TOPK", str(position))
    eng = Engine(model("tiny", "q8_0"))
    with pytest.raises(MgbError) as e:
        eng.log_softmax_topk(x, 4)
    assert e.value.code == _lib.MGB_ERR_CUDA
    assert "ran out of time" in str(e.value)
    eng.close()
    monkeypatch.delenv("MGB_TEST_WITHHOLD_TOPK")
    want_v, want_i = oracle.log_softmax_topk(x, 4)
    got_v, got_i = Engine(model("tiny", "q8_0")).log_softmax_topk(x, 4)
    np.testing.assert_array_equal(got_i, want_i)
    assert np.array_equal(got_v.view(np.uint32), want_v.view(np.uint32))


def test_beam_one_equals_greedy_on_device(gpu, model):
    """pipeline.rs:60-69: beam 1 gives the greedy output."""
    path = model("tiny", "q8_0")
    src = tiny_sentences()
    t = Translator(Engine(path))
    greedy = t.generate(src, TINY_TGT, GenOptions(max_new_tokens=16))
    eng = Engine(path)
    out, lens = eng.beam(eng.encode(src), TINY_TGT, 1, 16)
    assert [[int(x) for x in out[i, : lens[i]]] for i in range(len(src))] == greedy


@pytest.mark.parametrize("cluster", ["1", "2", "4"])
@pytest.mark.parametrize("n", [1, 6])
def test_small_batch_cluster_sizes_bit_exact(gpu, model, n, cluster, monkeypatch):
    """The small-batch matmuls share their input's q8_1 quantization across a
    cluster of CTAs (8 by default, MGB_SMALL_CLUSTER); every cluster size, and
    none, gives the oracle's tokens and logits bit for bit."""
    monkeypatch.setenv("MGB_SMALL_CLUSTER", cluster)
    monkeypatch.setenv("MGB_STEP_KERNEL", "0")
    path = model("wide", "q4_k_m")
    V = models.config_of("wide").vocab_size
    src = mid_sentences(V, n=n, seed=23)
    want_ids, want_logits = oracle.Oracle(path).greedy(src, V - 2, 4, force=True, logits=True)
    eng = Engine(path)
    got_ids, got_logits = eng.greedy_logits(eng.encode(src), V - 2, 4, force=True)
    np.testing.assert_array_equal(got_ids, want_ids)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32))


@pytest.mark.parametrize("step_kernel", ["1", "0"])
@pytest.mark.parametrize("preset", ["q4_k_m", "q8_0"])
@pytest.mark.parametrize("n", [1, 2, 3, 5, 8])
def test_small_batches_bit_exact(gpu, model, preset, n, step_kernel, monkeypatch):
    """1-8 rows run the reference's MMVQ arithmetic: the padded batch (1, 2, 4 or
    8 rows) picks candle's warp count (4 warps up to 4 rows, 2 for 5-8). Greedy
    steps run as the persistent step kernel (step_kernel 1) or one launch per
    operation (0); graph replay included; tokens and logits equal the oracle's
    bit for bit."""
    monkeypatch.setenv("MGB_STEP_KERNEL", step_kernel)
    path = model("mid", preset)
    V = models.config_of("mid").vocab_size
    src = mid_sentences(V, n=n, seed=21)
    want_ids, want_logits = oracle.Oracle(path).greedy(src, V - 2, 6, force=True, logits=True)
    eng = Engine(path)
    got_ids, got_logits = eng.greedy_logits(eng.encode(src), V - 2, 6, force=True)
    np.testing.assert_array_equal(got_ids, want_ids)
    assert np.array_equal(got_logits.view(np.uint32), want_logits.view(np.uint32)), \
        f"max |diff| {np.abs(got_logits - want_logits).max()}"
    out, _ = eng.greedy(eng.encode(src), V - 2, 6, force=True)  # CUDA-graph replay
    np.testing.assert_array_equal(out, want_ids)


def _bucket(n, lo, hi):
    """engine.cu bucket(): the next power of two >= max(n, lo), at most hi, at least n."""
    v = 1
    while v < max(n, lo):
        v <<= 1
    return max(min(v, hi), n)


@pytest.mark.parametrize("name,preset,n", [("wide", "q4_k_m", 1), ("wide", "q8_0", 3), ("wide", "q4_k_m", 40),
                                           ("mid", "q4_k_m", 6)])
def test_fast_vocab_shortlist_bit_exact(gpu, model_dir, name, preset, n):
    """--fast-vocab (model.rs:556-612, malaga.cu:280-326): the LM head over the
    shortlist's rows plus the source tokens' logits, the first maximum of the
    concatenated list mapped back to its token; tokens equal the oracle's."""
    cfg = models.config_of(name)
    V = cfg.vocab_size
    tgt = V - 2
    ids = models.synthetic_shortlist(V, V // 8, 9, [tgt])
    path = models.shortlist_model_path(name, preset, 0, {"xx_Test": ids}, model_dir)
    src = models.random_sources(n, 3, 20, V, 31, src_tag=V - 1)
    eng = Engine(path)
    sl = eng.shortlist("xx_Test")
    assert sl == 0 and eng.shortlist("yy_None") == -1
    got, _ = eng.greedy(eng.encode(src), tgt, 8, shortlist=sl)
    s_bucket = _bucket(max(len(r) for r in src), 16, cfg.max_position_embeddings)
    want = oracle.Oracle(path).greedy_shortlist(src, tgt, 8, ids, s_bucket)
    np.testing.assert_array_equal(got, want)
    # graph replay of the cached shortlist state
    again, _ = eng.greedy(eng.encode(src), tgt, 8, shortlist=sl)
    np.testing.assert_array_equal(again, want)


def test_fast_vocab_requires_the_start_tokens(gpu, model_dir):
    """translator.rs:186-192: a shortlist without the forced tokens is refused by
    the engine; Translator falls back to the full vocabulary."""
    V = models.config_of("mid").vocab_size
    ids = models.synthetic_shortlist(V, 200, 3, [])  # no target language token
    path = models.shortlist_model_path("mid", "q4_k_m", 0, {"zz_Test": ids}, model_dir)
    src = models.random_sources(2, 3, 10, V, 5, src_tag=V - 1)
    eng = Engine(path)
    with pytest.raises(MgbError):
        eng.greedy(eng.encode(src), V - 2, 4, shortlist=eng.shortlist("zz_Test"))
    t = Translator(eng)
    full = t.generate(src, V - 2, GenOptions(max_new_tokens=6))
    assert t.generate(src, V - 2, GenOptions(max_new_tokens=6, shortlist="zz_Test")) == full
