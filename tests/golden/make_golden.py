"""Generates the golden fixtures under tests/golden/ (run from the repo root):

    python tests/golden/make_golden.py

1. tiny_hf_greedy.npz — Hugging Face transformers' M2M100ForConditionalGeneration
   (the f32 semantics the reference claims parity with: spec/manual-tests.md
   MT-01, docs/performance.md "en f32, la sortie est identique à transformers")
   loaded with the reference's tiny test checkpoint (testutil.rs:16-101, seed 7)
   and run greedily, teacher-free, on the 6 sentences of pipeline.rs:132-134
   (fr -> mg). Stores source ids, generated ids and every step's logits.
2. dequant_golden.npz — gguf-py's dequantization of the Q8_0 / Q4_K / Q6_K
   blocks our converter writes for a seeded matrix (pins the block layouts).

Both are small; the tests compare the CPU oracle against them.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from malaga_b200 import convert as C  # noqa: E402
from malaga_b200 import gguf_io as G  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
SRC_LANG, TGT_LANG = 254, 256  # fra_Latn, plt_Latn in the tiny vocabulary
STEPS = 16


def tiny_sources() -> list[list[int]]:
    return [[SRC_LANG] + C.tiny_sentence(3 + 4 * i, i) + [2] for i in range(6)]


def hf_greedy():
    import torch
    from transformers import M2M100Config, M2M100ForConditionalGeneration

    cfg, get, _ = C.tiny_source(7)
    hc = M2M100Config(vocab_size=cfg.vocab_size, d_model=cfg.d_model, encoder_layers=cfg.encoder_layers,
                      decoder_layers=cfg.decoder_layers, encoder_attention_heads=cfg.encoder_attention_heads,
                      decoder_attention_heads=cfg.decoder_attention_heads, encoder_ffn_dim=cfg.encoder_ffn_dim,
                      decoder_ffn_dim=cfg.decoder_ffn_dim, max_position_embeddings=cfg.max_position_embeddings,
                      scale_embedding=True, activation_function="relu", dropout=0.0, attention_dropout=0.0,
                      activation_dropout=0.0, pad_token_id=1, bos_token_id=0, eos_token_id=2,
                      decoder_start_token_id=2, tie_word_embeddings=True)
    model = M2M100ForConditionalGeneration(hc).eval()
    sd = model.state_dict()
    new = {}
    for name in sd:
        if name in ("model.encoder.embed_tokens.weight", "model.decoder.embed_tokens.weight", "lm_head.weight"):
            src = "model.shared.weight"
        elif "embed_positions" in name:
            continue
        else:
            src = name
        new[name] = torch.from_numpy(np.array(get(src), dtype=np.float32))
    missing, unexpected = model.load_state_dict(new, strict=False)
    assert not unexpected and all("embed_positions" in m for m in missing), (missing, unexpected)

    src = tiny_sources()
    s = max(len(r) for r in src)
    ids = torch.full((len(src), s), 1, dtype=torch.long)
    mask = torch.zeros((len(src), s), dtype=torch.long)
    for i, r in enumerate(src):
        ids[i, : len(r)] = torch.tensor(r)
        mask[i, : len(r)] = 1
    dec = torch.tensor([[2, TGT_LANG]] * len(src))
    toks, logits = [], []
    with torch.no_grad():
        for _ in range(STEPS):
            out = model(input_ids=ids, attention_mask=mask, decoder_input_ids=dec).logits[:, -1].float()
            nxt = out.argmax(-1)
            toks.append(nxt.numpy())
            logits.append(out.numpy())
            dec = torch.cat([dec, nxt[:, None]], 1)
    np.savez_compressed(os.path.join(OUT, "tiny_hf_greedy.npz"),
                        src_ids=ids.numpy().astype(np.uint32), src_lens=mask.sum(1).numpy().astype(np.uint32),
                        tokens=np.stack(toks, 1).astype(np.uint32), logits=np.stack(logits, 0).astype(np.float32),
                        tgt=np.uint32(TGT_LANG))


def dequant_golden():
    from gguf import GGMLQuantizationType, quants

    x = C.seeded_normal(16 * 512, 11, 0, 0.02).reshape(16, 512)
    x[3, :256] = 0.0  # an all-zero super-block
    x[5, 40:72] *= 50.0  # a block with a large outlier range
    out = {"x": x}
    for t, name in ((G.Q8_0, "Q8_0"), (G.Q4_K, "Q4_K"), (G.Q6_K, "Q6_K")):
        q = C.quantize(x, t).reshape(16, -1)
        out[f"{name}_bytes"] = q
        out[f"{name}_deq"] = quants.dequantize(q, GGMLQuantizationType[name]).astype(np.float32)
    np.savez_compressed(os.path.join(OUT, "dequant_golden.npz"), **out)


if __name__ == "__main__":
    hf_greedy()
    dequant_golden()
    print("golden fixtures written to", OUT)
