"""Synthetic models and inputs of the benchmark configurations.

No checkpoint or dataset is available offline, so every model is random-init
from a seed with the NLLB-200 architecture of the configuration and converted
to GGUF by malaga_b200.convert (the reference's converter layout); inputs are
seeded uniform token ids with the configured length distributions.

Files are generated on first use into $MGB_MODEL_DIR (default /tmp/mgb_models)
and reused afterwards.
"""
from __future__ import annotations

import dataclasses
import os

import numpy as np

from . import convert as C

MODEL_DIR = os.environ.get("MGB_MODEL_DIR", "/tmp/mgb_models")

# Language tags of the synthetic large vocabulary (any in-vocabulary ids work
# with random weights; these sit in NLLB's language-code range).
SRC_TAG, TGT_TAG = 256047, 256147


def _mid(vocab=4000, d=256, heads=4, ffn=1024, layers=2, max_pos=256):
    return C.NllbConfig(vocab_size=vocab, d_model=d, encoder_layers=layers, decoder_layers=layers,
                        encoder_attention_heads=heads, decoder_attention_heads=heads, encoder_ffn_dim=ffn,
                        decoder_ffn_dim=ffn, max_position_embeddings=max_pos)


SPECS = {
    # name: (config, preset, seed, std)
    "mid": (_mid(), 0.05),
    "wide": (_mid(vocab=8192, d=1024, heads=16, ffn=4096, layers=2, max_pos=1024), 0.02),
    # the 3.3B layer shapes (d_model 2048, 16 heads of 128, FFN 8192) with 2+2 layers
    # and a smaller vocabulary, so that the CPU oracle checks them in seconds
    "3.3b-lite": (_mid(vocab=16384, d=2048, heads=16, ffn=8192, layers=2, max_pos=256), 0.02),
    # config 3's layer shapes (d_model 1024, FFN 8192, the full 256206 vocabulary) with 2+2 layers
    "1.3b-lite": (C.NllbConfig(vocab_size=256206, d_model=1024, encoder_layers=2, decoder_layers=2,
                               encoder_attention_heads=16, decoder_attention_heads=16, encoder_ffn_dim=8192,
                               decoder_ffn_dim=8192, max_position_embeddings=1024), 0.02),
    "600m": (C.NLLB_600M, 0.02),
    "1.3b": (C.NLLB_1_3B, 0.02),
    "3.3b": (C.NLLB_3_3B, 0.02),
}


def model_path(name: str, preset: str, seed: int = 0, directory: str | None = None) -> str:
    """Path of the GGUF for (architecture, preset, seed), generated on first use."""
    directory = directory or MODEL_DIR
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{name}-{preset}-s{seed}.gguf")
    if os.path.exists(path):
        return path
    if name == "tiny":
        cfg, get, tok = C.tiny_source(7 if seed == 0 else seed)
        C.convert(cfg, get, path, preset, "tiny", tok)
        return path
    cfg, std = SPECS[name]
    C.convert(cfg, C.random_init_source(cfg, seed, std), path, preset, f"synthetic-nllb-{name}")
    return path


def synthetic_shortlist(vocab: int, n: int, seed: int, keep: list[int]) -> list[int]:
    """A vocabulary shortlist for tests and benches: the special tokens 0-3 (kept by
    convert.rs:190), the ids in `keep` (language tokens) and n seeded ids."""
    ids = set(range(4)) | set(int(k) for k in keep)
    ids |= set(int(x) for x in C.seeded_uniform_u32(n, seed, 5, 4, vocab))
    return sorted(ids)


def shortlist_model_path(name: str, preset: str, seed: int, shortlists: dict[str, list[int]],
                         directory: str | None = None) -> str:
    """Path of the GGUF for (architecture, preset, seed) with vocabulary shortlists
    ({language code: ids}, --fast-vocab), generated on first use."""
    directory = directory or MODEL_DIR
    os.makedirs(directory, exist_ok=True)
    tag = "-".join(f"{k}{len(v)}" for k, v in sorted(shortlists.items()))
    path = os.path.join(directory, f"{name}-{preset}-s{seed}-sl-{tag}.gguf")
    if not os.path.exists(path):
        cfg, std = SPECS[name]
        C.convert(cfg, C.random_init_source(cfg, seed, std), path, preset, f"synthetic-nllb-{name}",
                  shortlists=shortlists)
    return path


def config_of(name: str) -> C.NllbConfig:
    return C.TINY if name == "tiny" else SPECS[name][0]


def random_sources(n: int, lo: int, hi: int, vocab: int, seed: int, src_tag: int = SRC_TAG, eos: int = 2,
                   fixed_len: int | None = None) -> list[list[int]]:
    """n sources `[src_tag] ids [eos]`, ids uniform in [4, vocab), body length uniform
    in [lo, hi] (or fixed_len), seeded."""
    lens = (np.full(n, fixed_len) if fixed_len is not None
            else C.seeded_uniform_u32(n, seed, 1, lo, hi + 1).astype(int))
    out = []
    for i in range(n):
        body = C.seeded_uniform_u32(int(lens[i]), seed, 1000 + i, 4, vocab)
        out.append([src_tag] + [int(x) for x in body] + [eos])
    return out


def poisson_arrivals(n: int, rate: float, seed: int) -> np.ndarray:
    """Arrival times (s) of a Poisson process of `rate` requests/s, seeded."""
    u = C.seeded_uniform_u32(n, seed, 3, 1, 1 << 24).astype(np.float64) / float(1 << 24)
    return np.cumsum(-np.log(u) / rate)


def lognormal_sources(n: int, median: float, lo: int, hi: int, vocab: int, seed: int) -> list[list[int]]:
    """Lengths lognormal(median, sigma 0.5) clipped to [lo, hi] (configs 4 and 5)."""
    z = C.seeded_normal(n, seed, 2, 1.0).astype(np.float64)
    lens = np.clip(np.round(median * np.exp(0.5 * z)), lo, hi).astype(int)
    return [random_sources(1, 0, 0, vocab, seed * 100000 + i, fixed_len=int(lens[i]))[0] for i in range(n)]


@dataclasses.dataclass
class Workload:
    name: str
    model: str
    preset: str
    seed: int
    batch: int
    steps: int
    sources: list


def workload(key: str) -> Workload:
    """The benchmark configurations as concrete inputs."""
    V = C.NLLB_600M.vocab_size
    if key == "c1":  # 600M q4_k_m, b1, 32-token source, 32 forced steps
        return Workload("c1", "600m", "q4_k_m", 0, 1, 32, random_sources(1, 32, 32, V, 0, fixed_len=32))
    if key == "c2":  # 600M q8_0, b64, lengths U[8,64], 64 forced steps
        src = sorted(random_sources(64, 8, 64, V, 1), key=len, reverse=True)
        return Workload("c2", "600m", "q8_0", 1, 64, 64, src)
    if key == "c2q4":  # the headline metric's q4_k_m weights on config 2's batch
        src = sorted(random_sources(64, 8, 64, V, 1), key=len, reverse=True)
        return Workload("c2q4", "600m", "q4_k_m", 0, 64, 64, src)
    if key == "c5":  # server simulation: 4096 single-sentence requests, lengths lognormal(24), 4..96
        return Workload("c5", "600m", "q4_k_m", 0, 64, 0, lognormal_sources(4096, 24, 4, 96, V, 4))
    if key == "c3":  # 1.3B q4_k_m (seed 2), beam 4 over 16 sources of 48 tokens, at most 96 steps
        return Workload("c3", "1.3b", "q4_k_m", 2, 16, 96, random_sources(16, 48, 48, V, 2, fixed_len=48))
    if key == "c4":  # 3.3B q4_k_m (seed 3), 1024 sentences lognormal(28) clipped 8..128, batches of 128,
        # 128 forced steps, partitioned over the GPUs like dp600
        return Workload("c4", "3.3b", "q4_k_m", 3, 128, 128, lognormal_sources(1024, 28, 8, 128, V, 3))
    if key == "dp600":  # the headline set: 1024 sentences (config 2's lengths) in batches of 64,
        # partitioned over the GPUs (translator.rs:140-147 batching, LPT placement)
        return Workload("dp600", "600m", "q4_k_m", 0, 64, 64, random_sources(1024, 8, 64, V, 1))
    raise KeyError(key)
