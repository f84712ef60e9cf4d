"""CPU: the converter writes malaga's GGUF layout (convert.rs:196-319, config.rs:71-113)."""
import numpy as np
import pytest

from malaga_b200 import convert as C
from malaga_b200 import gguf_io as G
from malaga_b200 import models


def test_metadata_keys_match_config_rs(model):
    meta, infos = G.read_metadata(model("tiny", "q8_0"))
    cfg = C.TINY
    assert meta["general.architecture"] == "nllb"
    assert meta["general.name"] == "tiny"
    assert meta["general.file_type"] == "q8_0"
    assert meta["tokenizer.ggml.model"] == "nllb"
    assert "WordLevel" in meta["tokenizer.huggingface.json"]
    expect = {"nllb.vocab_size": cfg.vocab_size, "nllb.embedding_length": 64, "nllb.encoder.block_count": 2,
              "nllb.decoder.block_count": 2, "nllb.encoder.attention.head_count": 4,
              "nllb.decoder.attention.head_count": 4, "nllb.encoder.feed_forward_length": 128,
              "nllb.decoder.feed_forward_length": 128, "nllb.context_length": 128, "nllb.scale_embedding": True,
              "nllb.max_length": 64, "tokenizer.ggml.bos_token_id": 0, "tokenizer.ggml.padding_token_id": 1,
              "tokenizer.ggml.eos_token_id": 2, "tokenizer.ggml.decoder_start_token_id": 2}
    for k, v in expect.items():
        assert meta[k] == v, k


def test_gguf_py_reads_our_files(model):
    """An independent reader (gguf-py) parses the file and agrees on shapes and types."""
    from gguf import GGUFReader

    path = model("mid", "q4_k_m")
    r = GGUFReader(path)
    _, infos = G.read_metadata(path)
    assert len(r.tensors) == len(infos)
    for t in r.tensors:
        shape, ty, _ = infos[t.name]
        assert int(t.tensor_type) == ty
        assert tuple(int(x) for x in reversed(t.shape.tolist())) == shape


def test_preset_types_and_fallback(model):
    """q4_k_m: linears Q4_K, ffn_down and the embedding Q6_K, norms/biases F32
    (convert.rs:67-91); rows that are not whole k-quant blocks fall back to Q8_0
    (convert.rs:150-162) — every matrix of the tiny model."""
    _, infos = G.read_metadata(model("mid", "q4_k_m"))
    assert infos["token_embd.weight"][1] == G.Q6_K
    assert infos["dec.blk.0.attn_qkv.weight"][1] == G.Q4_K
    assert infos["dec.blk.0.cross_attn_kv.weight"][1] == G.Q4_K
    assert infos["dec.blk.1.ffn_down.weight"][1] == G.Q6_K
    assert infos["enc.blk.0.ffn_up.weight"][1] == G.Q4_K
    assert infos["dec.blk.0.attn_qkv.bias"][1] == G.F32
    assert infos["enc.output_norm.weight"][1] == G.F32
    _, tiny = G.read_metadata(model("tiny", "q4_k_m"))
    assert {t for n, (_, t, _) in tiny.items() if n.endswith(".weight") and "norm" not in n} == {G.Q8_0}
    assert C.fallback_dtype(G.Q4_K, (10, 512)) == G.Q4_K
    assert C.fallback_dtype(G.Q4_K, (10, 96)) == G.Q8_0
    assert C.fallback_dtype(G.Q8_0, (10, 40)) == G.F16
    assert C.fallback_dtype(G.Q4_K, (512,)) == G.F32


def test_tensor_layout_fused_and_prescaled(model):
    """attn_qkv = cat(q*s, k, v), cross_attn_kv = cat(k, v), q bias pre-scaled
    (convert.rs:242-267), checked on the exact f32 preset."""
    import oracle

    cfg, get, _ = C.tiny_source(7)
    orc = oracle.Oracle(model("tiny", "f32"))
    d, s = cfg.d_model, np.float32((cfg.d_model // cfg.decoder_attention_heads) ** -0.5)
    p = "model.decoder.layers.1"
    qw = get(f"{p}.self_attn.q_proj.weight") * s
    kw = get(f"{p}.self_attn.k_proj.weight")
    for r, c in ((0, 0), (5, 17), (63, 63)):
        assert orc.dequant("dec.blk.1.attn_qkv.weight", r, c) == qw[r, c]
        assert orc.dequant("dec.blk.1.attn_qkv.weight", d + r, c) == kw[r, c]
    vw = get(f"{p}.encoder_attn.v_proj.weight")
    assert orc.dequant("dec.blk.1.cross_attn_kv.weight", d + 3, 9) == vw[3, 9]


def test_tiny_source_matches_testutil_recipe():
    """testutil.rs:57-69: first draws of xorshift64 seeded 7 (|1), scale 0.5 for the embedding."""
    cfg, get, _ = C.tiny_source(7)
    emb = get("model.shared.weight")
    assert emb.shape == (257, 64) and emb.dtype == np.float32
    s = ((7 * 0x9E3779B97F4A7C15) & (2**64 - 1)) | 1
    M = 2**64 - 1
    s ^= (s << 13) & M
    s ^= s >> 7
    s ^= (s << 17) & M
    v = (np.float32(s >> 40) / np.float32(1 << 24) - np.float32(0.5)) * np.float32(2.0) * np.float32(0.5)
    assert emb[0, 0] == v
    assert np.abs(emb).max() <= 0.5


def test_workloads_match_baseline_configs():
    w = models.workload("c2")
    assert len(w.sources) == 64 and w.steps == 64
    body = [len(s) - 2 for s in w.sources]
    assert min(body) >= 8 and max(body) <= 64
    assert [len(s) for s in w.sources] == sorted([len(s) for s in w.sources], reverse=True)
    assert all(4 <= t < 256206 for s in w.sources for t in s[1:-1])
    c1 = models.workload("c1")
    assert len(c1.sources) == 1 and len(c1.sources[0]) == 34 and c1.steps == 32


def test_shortlist_metadata_and_reduced_head(model_dir):
    """--fast-vocab shortlists (convert.rs:218-232): nllb.shortlist.<code> holds the
    sorted ids, lm_head.<code>.weight the embedding rows of those ids, quantized
    like the embedding (so its bytes are the embedding's rows)."""
    from gguf import GGUFReader

    V = models.config_of("mid").vocab_size
    ids = models.synthetic_shortlist(V, 300, 7, [V - 2])
    path = models.shortlist_model_path("mid", "q4_k_m", 0, {"xx_Test": ids}, model_dir)
    meta, infos = G.read_metadata(path)
    assert meta["nllb.shortlist.xx_Test"] == ids
    d = models.config_of("mid").d_model
    shape, ty, _ = infos["lm_head.xx_Test.weight"]
    assert shape == (len(ids), d) and ty == infos["token_embd.weight"][1]
    r = GGUFReader(path)
    t = {x.name: np.asarray(x.data) for x in r.tensors}
    emb, head = t["token_embd.weight"], t["lm_head.xx_Test.weight"]
    assert np.array_equal(head.reshape(len(ids), -1), emb.reshape(V, -1)[ids])
