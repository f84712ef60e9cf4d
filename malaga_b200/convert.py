"""Hugging Face NLLB/M2M100 weights -> GGUF, following malaga's converter.

Restates crates/malaga-core/src/convert.rs:196-319 (tensor names, QKV fusion,
1/sqrt(head_dim) pre-scaling of the query weight and bias, fused cross K/V,
f32 norms/biases, metadata) and config.rs:60-113 (the ``nllb.*`` and
``tokenizer.ggml.*`` keys). Presets and per-tensor types follow
convert.rs:31-91; the k-quant fallback follows convert.rs:150-162.

The tensor *source* is a callable ``get(hf_name) -> np.float32 array``: a real
checkpoint, the tiny test model of crates/malaga-core/src/testutil.rs:16-101,
or the seeded random-init models of the benchmark configurations.
"""
from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass, field, asdict
from typing import Callable

import numpy as np

from . import gguf_io as G

ARCH = "nllb"
_HERE = os.path.dirname(os.path.abspath(__file__))


@dataclass
class NllbConfig:
    """Hyper-parameters (crates/malaga-core/src/config.rs:15-35)."""

    vocab_size: int
    d_model: int
    encoder_layers: int
    decoder_layers: int
    encoder_attention_heads: int
    decoder_attention_heads: int
    encoder_ffn_dim: int
    decoder_ffn_dim: int
    max_position_embeddings: int
    scale_embedding: bool = True
    bos_token_id: int = 0
    pad_token_id: int = 1
    eos_token_id: int = 2
    decoder_start_token_id: int = 2
    max_length: int = 200

    def to_gguf(self) -> list:
        u, k = G.U32, (lambda s: f"{ARCH}.{s}")
        return [
            (k("vocab_size"), u(self.vocab_size)),
            (k("embedding_length"), u(self.d_model)),
            (k("encoder.block_count"), u(self.encoder_layers)),
            (k("decoder.block_count"), u(self.decoder_layers)),
            (k("encoder.attention.head_count"), u(self.encoder_attention_heads)),
            (k("decoder.attention.head_count"), u(self.decoder_attention_heads)),
            (k("encoder.feed_forward_length"), u(self.encoder_ffn_dim)),
            (k("decoder.feed_forward_length"), u(self.decoder_ffn_dim)),
            (k("context_length"), u(self.max_position_embeddings)),
            (k("scale_embedding"), G.Bool(self.scale_embedding)),
            (k("max_length"), u(self.max_length)),
            ("tokenizer.ggml.bos_token_id", u(self.bos_token_id)),
            ("tokenizer.ggml.padding_token_id", u(self.pad_token_id)),
            ("tokenizer.ggml.eos_token_id", u(self.eos_token_id)),
            ("tokenizer.ggml.decoder_start_token_id", u(self.decoder_start_token_id)),
        ]


# Architectures of the benchmark configurations (NLLB-200 model cards) and of
# the reference's tiny test model (testutil.rs:16-30).
TINY = NllbConfig(vocab_size=4 + 250 + 3, d_model=64, encoder_layers=2, decoder_layers=2,
                  encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=128,
                  decoder_ffn_dim=128, max_position_embeddings=128, max_length=64)
NLLB_600M = NllbConfig(vocab_size=256206, d_model=1024, encoder_layers=12, decoder_layers=12,
                       encoder_attention_heads=16, decoder_attention_heads=16, encoder_ffn_dim=4096,
                       decoder_ffn_dim=4096, max_position_embeddings=1024)
NLLB_1_3B = NllbConfig(vocab_size=256206, d_model=1024, encoder_layers=24, decoder_layers=24,
                       encoder_attention_heads=16, decoder_attention_heads=16, encoder_ffn_dim=8192,
                       decoder_ffn_dim=8192, max_position_embeddings=1024)
NLLB_3_3B = NllbConfig(vocab_size=256206, d_model=2048, encoder_layers=24, decoder_layers=24,
                       encoder_attention_heads=16, decoder_attention_heads=16, encoder_ffn_dim=8192,
                       decoder_ffn_dim=8192, max_position_embeddings=1024)

# Preset -> (linear type, ffn_down type, embedding type): convert.rs:67-91.
PRESETS = {
    "f32": (G.F32, G.F32, G.F32),
    "q8_0": (G.Q8_0, G.Q8_0, G.Q8_0),
    "q6_k": (G.Q6_K, G.Q6_K, G.Q6_K),
    "q4_k_m": (G.Q4_K, G.Q6_K, G.Q6_K),
}


def fallback_dtype(t: int, shape: tuple[int, ...]) -> int:
    """convert.rs:150-162: 1-D -> F32; k-quants need rows % 256, else Q8_0 (rows % 32), else F16."""
    if len(shape) < 2:
        return G.F32
    row = shape[-1]
    blk = G.BLOCK[t][0]
    if row % blk == 0:
        return t
    if row % 32 == 0:
        return G.Q8_0
    return G.F16


_lib = None


def _convert_lib():
    global _lib
    if _lib is None:
        path = os.path.join(_HERE, "libmgb_convert.so")
        if not os.path.exists(path):
            from .build import build_convert
            build_convert()
        lib = ctypes.CDLL(path)
        lib.mgbc_quantize.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_long, ctypes.c_long, ctypes.c_void_p]
        lib.mgbc_quantize.restype = ctypes.c_int
        lib.mgbc_normal.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float]
        lib.mgbc_uniform_u32.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_uint64, ctypes.c_uint64,
                                         ctypes.c_uint32, ctypes.c_uint32]
        _lib = lib
    return _lib


def quantize(x: np.ndarray, t: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    rows = x.size // n
    out = np.empty(rows * G.row_bytes(t, n), np.uint8)
    if _convert_lib().mgbc_quantize(t, x.ctypes.data, rows, n, out.ctypes.data) != 0:
        raise ValueError(f"cannot quantize rows of {n} values to {G.TYPE_NAMES[t]}")
    return out


def seeded_normal(n: int, seed: int, stream: int, std: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    _convert_lib().mgbc_normal(out.ctypes.data, n, seed, stream, std)
    return out


def seeded_uniform_u32(n: int, seed: int, stream: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    _convert_lib().mgbc_uniform_u32(out.ctypes.data, n, seed, stream, lo, hi)
    return out


def _tokenizer_json(cfg: NllbConfig, langs: list[str], words: int) -> str:
    specials = ["<s>", "<pad>", "</s>", "<unk>"]
    vocab = {s: i for i, s in enumerate(specials)}
    added = [{"id": i, "content": s, "single_word": False, "lstrip": False, "rstrip": False,
              "normalized": False, "special": True} for i, s in enumerate(specials)]
    for w in range(words):
        vocab[f"w{w}"] = len(specials) + w
    for i, lang in enumerate(langs):
        tid = cfg.vocab_size - len(langs) + i
        vocab[lang] = tid
        added.append({"id": tid, "content": lang, "single_word": False, "lstrip": False, "rstrip": False,
                      "normalized": False, "special": True})
    return json.dumps({"version": "1.0", "truncation": None, "padding": None, "added_tokens": added,
                       "normalizer": None, "pre_tokenizer": {"type": "Whitespace"}, "post_processor": None,
                       "decoder": None, "model": {"type": "WordLevel", "vocab": vocab, "unk_token": "<unk>"}})


def convert(cfg: NllbConfig, get: Callable[[str], np.ndarray], out: str, preset: str = "q4_k_m",
            name: str = "nllb", tokenizer_json: str | None = None,
            shortlists: dict[str, list[int]] | None = None) -> None:
    """Writes the GGUF file of convert.rs:196-319 from HF-named f32 tensors.

    shortlists: {language code: vocabulary ids} for `--fast-vocab` decoding
    (convert.rs:218-232): each is stored sorted as `nllb.shortlist.<code>` with
    its reduced LM head `lm_head.<code>.weight` (the embedding rows of those ids,
    quantized like the embedding). The reference builds the ids from a corpus
    with the tokenizer and adds the language token; callers pass the ids."""
    lin, down, emb = PRESETS[preset]
    enc_s = np.float32((cfg.d_model // cfg.encoder_attention_heads) ** -0.5)
    dec_s = np.float32((cfg.d_model // cfg.decoder_attention_heads) ** -0.5)
    plans: list[G.TensorPlan] = []

    def add(gname: str, shape: tuple[int, ...], t: int, make: Callable[[], np.ndarray]):
        t = fallback_dtype(t, shape)
        plans.append(G.TensorPlan(gname, shape, t, lambda: quantize(make(), t)))

    d, V = cfg.d_model, cfg.vocab_size
    add("token_embd.weight", (V, d), emb, lambda: get("model.shared.weight"))
    sl_meta = []
    for code, ids in (shortlists or {}).items():
        ids = sorted({int(i) for i in ids})
        if not ids or ids[0] < 0 or ids[-1] >= V:
            raise ValueError(f"shortlist {code}: ids outside the vocabulary")
        idx = np.array(ids, np.int64)
        add(f"lm_head.{code}.weight", (len(ids), d), emb, lambda idx=idx: get("model.shared.weight")[idx])
        sl_meta.append((f"{ARCH}.shortlist.{code}", ids))
    for side, n_layers, s, ffn in (("encoder", cfg.encoder_layers, enc_s, cfg.encoder_ffn_dim),
                                   ("decoder", cfg.decoder_layers, dec_s, cfg.decoder_ffn_dim)):
        short = side[:3]
        for i in range(n_layers):
            p, o = f"model.{side}.layers.{i}", f"{short}.blk.{i}"

            def qkv_w(p=p, s=s):
                return np.concatenate([get(f"{p}.self_attn.q_proj.weight") * s, get(f"{p}.self_attn.k_proj.weight"),
                                       get(f"{p}.self_attn.v_proj.weight")], 0)

            def qkv_b(p=p, s=s):
                return np.concatenate([get(f"{p}.self_attn.q_proj.bias") * s, get(f"{p}.self_attn.k_proj.bias"),
                                       get(f"{p}.self_attn.v_proj.bias")], 0)

            add(f"{o}.attn_qkv.weight", (3 * d, d), lin, qkv_w)
            add(f"{o}.attn_qkv.bias", (3 * d,), G.F32, qkv_b)
            add(f"{o}.attn_out.weight", (d, d), lin, lambda p=p: get(f"{p}.self_attn.out_proj.weight"))
            add(f"{o}.attn_out.bias", (d,), G.F32, lambda p=p: get(f"{p}.self_attn.out_proj.bias"))
            add(f"{o}.attn_norm.weight", (d,), G.F32, lambda p=p: get(f"{p}.self_attn_layer_norm.weight"))
            add(f"{o}.attn_norm.bias", (d,), G.F32, lambda p=p: get(f"{p}.self_attn_layer_norm.bias"))
            if side == "decoder":
                add(f"{o}.cross_attn_q.weight", (d, d), lin,
                    lambda p=p, s=s: get(f"{p}.encoder_attn.q_proj.weight") * s)
                add(f"{o}.cross_attn_q.bias", (d,), G.F32, lambda p=p, s=s: get(f"{p}.encoder_attn.q_proj.bias") * s)
                add(f"{o}.cross_attn_kv.weight", (2 * d, d), lin,
                    lambda p=p: np.concatenate([get(f"{p}.encoder_attn.k_proj.weight"),
                                                get(f"{p}.encoder_attn.v_proj.weight")], 0))
                add(f"{o}.cross_attn_kv.bias", (2 * d,), G.F32,
                    lambda p=p: np.concatenate([get(f"{p}.encoder_attn.k_proj.bias"),
                                                get(f"{p}.encoder_attn.v_proj.bias")], 0))
                add(f"{o}.cross_attn_out.weight", (d, d), lin, lambda p=p: get(f"{p}.encoder_attn.out_proj.weight"))
                add(f"{o}.cross_attn_out.bias", (d,), G.F32, lambda p=p: get(f"{p}.encoder_attn.out_proj.bias"))
                add(f"{o}.cross_attn_norm.weight", (d,), G.F32,
                    lambda p=p: get(f"{p}.encoder_attn_layer_norm.weight"))
                add(f"{o}.cross_attn_norm.bias", (d,), G.F32, lambda p=p: get(f"{p}.encoder_attn_layer_norm.bias"))
            add(f"{o}.ffn_up.weight", (ffn, d), lin, lambda p=p: get(f"{p}.fc1.weight"))
            add(f"{o}.ffn_up.bias", (ffn,), G.F32, lambda p=p: get(f"{p}.fc1.bias"))
            add(f"{o}.ffn_down.weight", (d, ffn), down, lambda p=p: get(f"{p}.fc2.weight"))
            add(f"{o}.ffn_down.bias", (d,), G.F32, lambda p=p: get(f"{p}.fc2.bias"))
            add(f"{o}.ffn_norm.weight", (d,), G.F32, lambda p=p: get(f"{p}.final_layer_norm.weight"))
            add(f"{o}.ffn_norm.bias", (d,), G.F32, lambda p=p: get(f"{p}.final_layer_norm.bias"))
        add(f"{short}.output_norm.weight", (d,), G.F32, lambda side=side: get(f"model.{side}.layer_norm.weight"))
        add(f"{short}.output_norm.bias", (d,), G.F32, lambda side=side: get(f"model.{side}.layer_norm.bias"))

    if tokenizer_json is None:
        tokenizer_json = _tokenizer_json(cfg, [], 0)
    meta = [
        ("general.architecture", ARCH),
        ("general.name", name),
        ("general.file_type", preset),
        ("general.license", "cc-by-nc-4.0"),
        ("general.source.url", f"https://huggingface.co/{name}"),
        ("tokenizer.ggml.model", "nllb"),
        ("tokenizer.huggingface.json", tokenizer_json),
    ] + cfg.to_gguf() + sl_meta
    tmp = out + ".partial"
    G.write_gguf(tmp, meta, plans)
    os.replace(tmp, out)


# ---------------------------------------------------------------------------
# Tensor sources


def hf_shapes(cfg: NllbConfig) -> dict[str, tuple[int, ...]]:
    d = cfg.d_model
    shapes = {"model.shared.weight": (cfg.vocab_size, d)}
    for side, n_layers, ffn in (("encoder", cfg.encoder_layers, cfg.encoder_ffn_dim),
                                ("decoder", cfg.decoder_layers, cfg.decoder_ffn_dim)):
        for i in range(n_layers):
            p = f"model.{side}.layers.{i}"
            attns = ["self_attn"] + (["encoder_attn"] if side == "decoder" else [])
            for a in attns:
                for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
                    shapes[f"{p}.{a}.{proj}.weight"] = (d, d)
                    shapes[f"{p}.{a}.{proj}.bias"] = (d,)
                shapes[f"{p}.{a}_layer_norm.weight"] = (d,)
                shapes[f"{p}.{a}_layer_norm.bias"] = (d,)
            shapes[f"{p}.fc1.weight"] = (ffn, d)
            shapes[f"{p}.fc1.bias"] = (ffn,)
            shapes[f"{p}.fc2.weight"] = (d, ffn)
            shapes[f"{p}.fc2.bias"] = (d,)
            shapes[f"{p}.final_layer_norm.weight"] = (d,)
            shapes[f"{p}.final_layer_norm.bias"] = (d,)
        shapes[f"model.{side}.layer_norm.weight"] = (d,)
        shapes[f"model.{side}.layer_norm.bias"] = (d,)
    return shapes


def random_init_source(cfg: NllbConfig, seed: int, std: float = 0.02) -> Callable[[str], np.ndarray]:
    """Seeded random init with the M2M100 initialisation rule: matrices and the
    embedding N(0, std) (embedding row `pad` zeroed), biases 0, LayerNorm
    gamma=1 / beta=0. Each tensor draws from its own stream (its index in the
    checkpoint), so any tensor can be regenerated on its own."""
    shapes = hf_shapes(cfg)
    index = {n: i for i, n in enumerate(shapes)}

    def get(name: str) -> np.ndarray:
        shape = shapes[name]
        if name.endswith("layer_norm.weight"):
            return np.ones(shape, np.float32)
        if len(shape) == 1:
            return np.zeros(shape, np.float32)
        w = seeded_normal(int(np.prod(shape)), seed, index[name], std).reshape(shape)
        if name == "model.shared.weight":
            w[cfg.pad_token_id] = 0.0
        return w

    return get


def tiny_source(seed: int = 7) -> tuple[NllbConfig, Callable[[str], np.ndarray], str]:
    """The reference's tiny checkpoint (testutil.rs:16-101): xorshift64 weights
    drawn in the file's insertion order, uniform in [-scale, scale)."""
    cfg = TINY
    d, ffn, layers, V = cfg.d_model, cfg.decoder_ffn_dim, cfg.encoder_layers, cfg.vocab_size
    M = (1 << 64) - 1
    state = [((seed * 0x9E3779B97F4A7C15) & M) | 1]

    def rand(shape, scale):
        n = int(np.prod(shape))
        vals = np.empty(n, np.uint32)
        s = state[0]
        for i in range(n):
            s ^= (s << 13) & M
            s ^= s >> 7
            s ^= (s << 17) & M
            vals[i] = s >> 40
        state[0] = s
        f = vals.astype(np.float32) / np.float32(1 << 24) - np.float32(0.5)
        return ((f * np.float32(2.0)) * np.float32(scale)).reshape(shape)

    w = {"model.shared.weight": rand((V, d), 0.5)}
    ones, zeros = np.ones(d, np.float32), np.zeros(d, np.float32)
    for side in ("encoder", "decoder"):
        for l in range(layers):
            p = f"model.{side}.layers.{l}"
            for a in ["self_attn"] + (["encoder_attn"] if side == "decoder" else []):
                for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
                    w[f"{p}.{a}.{proj}.weight"] = rand((d, d), 0.3)
                    w[f"{p}.{a}.{proj}.bias"] = rand((d,), 0.1)
                w[f"{p}.{a}_layer_norm.weight"] = ones
                w[f"{p}.{a}_layer_norm.bias"] = zeros
            w[f"{p}.fc1.weight"] = rand((ffn, d), 0.3)
            w[f"{p}.fc1.bias"] = rand((ffn,), 0.1)
            w[f"{p}.fc2.weight"] = rand((d, ffn), 0.3)
            w[f"{p}.fc2.bias"] = rand((d,), 0.1)
            w[f"{p}.final_layer_norm.weight"] = ones
            w[f"{p}.final_layer_norm.bias"] = zeros
        w[f"model.{side}.layer_norm.weight"] = ones
        w[f"model.{side}.layer_norm.bias"] = zeros
    tok = _tokenizer_json(cfg, ["fra_Latn", "eng_Latn", "plt_Latn"], 250)
    return cfg, w.__getitem__, tok


def tiny_sentence(n: int, seed: int) -> list[int]:
    """Token ids of testutil.rs:104-106 `sentence(n, seed)` (word w_k has id 4+k)."""
    return [4 + (seed * 31 + i * 17) % 250 for i in range(n)]
