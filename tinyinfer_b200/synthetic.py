"""Seeded synthetic models and inputs for the MiniPrefix 135M-shape Llama.

Weights follow the MPFX0001 orientation that MiniPrefix loads
(miniprefix/src/model/model.cpp:28-38 in TinyInfer v0.3.0): every 2-D linear is
stored [in, out], the embedding [vocab, hidden], RMSNorm weights [hidden].
Values are N(0, std) float32 from numpy's PCG64 with a recorded seed; RMSNorm
weights are 1, as in the reference's own regression model
(miniprefix/tests/cow_test.cpp:124).
"""
from __future__ import annotations

from dataclasses import dataclass, asdict

import numpy as np


@dataclass(frozen=True)
class ModelConfig:
    """Mirror of miniprefix::ModelConfig (miniprefix/include/miniprefix/model.h:9-16)."""

    layers: int = 30
    hidden: int = 576
    intermediate: int = 1536
    heads: int = 9
    kv_heads: int = 3
    vocabulary: int = 49152
    context: int = 8192
    eos: int = 0
    rms_epsilon: float = 1e-5
    rope_theta: float = 1e5
    tied: bool = True

    @property
    def head_dimension(self) -> int:
        return self.hidden // self.heads

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dimension

    def validate(self) -> None:
        """ModelConfig::validate (miniprefix/src/model/model.cpp:9-15)."""
        c = self
        bad = (c.layers < 1 or c.layers > 128 or c.hidden < 2 or c.hidden > 8192 or c.intermediate < 1
               or c.intermediate > 65536 or c.heads < 1 or c.kv_heads < 1 or c.hidden % c.heads
               or c.heads % c.kv_heads or (c.hidden // c.heads) % 2 or c.hidden // c.heads > 256
               or c.vocabulary < 2 or c.vocabulary > 262144 or c.context < 1 or c.context > 131072
               or c.eos < 0 or c.eos >= c.vocabulary or not np.isfinite(c.rms_epsilon) or c.rms_epsilon <= 0
               or not np.isfinite(c.rope_theta) or c.rope_theta <= 1)
        if bad:
            raise ValueError("unsupported/invalid Llama configuration")

    def as_dict(self) -> dict:
        return asdict(self)


SMOLLM2_135M = ModelConfig()


def tensor_names(c: ModelConfig) -> list[tuple[str, tuple[int, ...]]]:
    """Expected tensor names and shapes (model.cpp:28-38)."""
    out = [("model.embed_tokens.weight", (c.vocabulary, c.hidden)), ("model.norm.weight", (c.hidden,))]
    if not c.tied:
        out.append(("lm_head.weight", (c.hidden, c.vocabulary)))
    for l in range(c.layers):
        p = f"model.layers.{l}."
        out += [
            (p + "input_layernorm.weight", (c.hidden,)),
            (p + "post_attention_layernorm.weight", (c.hidden,)),
            (p + "self_attn.q_proj.weight", (c.hidden, c.hidden)),
            (p + "self_attn.k_proj.weight", (c.hidden, c.kv_width)),
            (p + "self_attn.v_proj.weight", (c.hidden, c.kv_width)),
            (p + "self_attn.o_proj.weight", (c.hidden, c.hidden)),
            (p + "mlp.gate_proj.weight", (c.hidden, c.intermediate)),
            (p + "mlp.up_proj.weight", (c.hidden, c.intermediate)),
            (p + "mlp.down_proj.weight", (c.intermediate, c.hidden)),
        ]
    return out


def random_weights(c: ModelConfig, seed: int = 0, std: float = 0.02) -> dict[str, np.ndarray]:
    """N(0, std) float32 linears/embedding, unit RMSNorm weights, PCG64(seed)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    weights = {}
    for name, shape in tensor_names(c):
        if name.endswith("norm.weight"):
            weights[name] = np.ones(shape, dtype=np.float32)
        else:
            a = rng.standard_normal(size=shape, dtype=np.float32)
            a *= np.float32(std)
            weights[name] = a
    return weights


def sine_weights(c: ModelConfig) -> dict[str, np.ndarray]:
    """The reference regression model's weights: 0.15*sin(k) with a running k over
    tensors in creation order, norms 1 (miniprefix/tests/cow_test.cpp:118-137)."""
    order = ["model.embed_tokens.weight"]
    if not c.tied:
        order.append("lm_head.weight")
    order.append("model.norm.weight")
    for l in range(c.layers):
        p = f"model.layers.{l}."
        order += [p + "input_layernorm.weight", p + "post_attention_layernorm.weight",
                  p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight",
                  p + "self_attn.o_proj.weight", p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight",
                  p + "mlp.down_proj.weight"]
    shapes = dict(tensor_names(c))
    seed = 0
    out = {}
    for name in order:
        shape = shapes[name]
        n = int(np.prod(shape))
        if name.endswith("norm.weight"):
            out[name] = np.ones(shape, dtype=np.float32)
        else:
            k = np.arange(seed + 1, seed + n + 1, dtype=np.float32)
            out[name] = (np.float32(0.15) * np.sin(k).astype(np.float32)).astype(np.float32).reshape(shape)
            seed += n
    return out


def random_tokens(count: int, vocabulary: int, seed: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(0, vocabulary, size=count, dtype=np.int64).astype(np.int32)


@dataclass(frozen=True)
class PrefixTreeRequest:
    root: int          # prefix-tree root the prompt starts from (routing key)
    path: tuple        # child index at each depth below the root (may be empty)
    prompt: np.ndarray  # int32 token ids
    max_new_tokens: int


def prefix_tree_requests(seed: int = 5, count: int = 2048, roots: int = 16, root_tokens: int = 2048,
                         branching: int = 4, depth: int = 3, segment: int = 256, min_len: int = 512,
                         max_len: int = 8192, min_new: int = 32, max_new: int = 512,
                         vocabulary: int = 49152) -> list[PrefixTreeRequest]:
    """Seeded requests drawn from a prefix tree (BASELINE config 5's workload).

    The tree: `roots` random root sequences of `root_tokens` tokens; every node
    has `branching` children, each adding its own random `segment`-token
    segment, down to `depth` levels (4 + 16 + 64 descendant paths per root at the
    defaults). A request picks a root and a depth uniformly, then a node at that
    depth uniformly; its path tokens are the root followed by the segments down
    to the node. The prompt length is uniform in [min_len, max_len]: a path
    longer than that is truncated, a shorter one is extended with tokens unique
    to the request. Decode lengths are uniform in [min_new, max_new].
    Segments are derived from (seed, root, path) alone, so the same node yields
    the same tokens in every request and on every rank.
    """
    rng = np.random.Generator(np.random.PCG64(seed))
    cache: dict = {}

    def tokens(root: int, path: tuple) -> np.ndarray:
        key = (root, path)
        if key not in cache:
            n = root_tokens if not path else segment
            g = np.random.Generator(np.random.PCG64([seed, 1 + root, len(path), *path]))
            cache[key] = g.integers(0, vocabulary, size=n, dtype=np.int64).astype(np.int32)
        return cache[key]

    out = []
    for i in range(count):
        root = int(rng.integers(0, roots))
        d = int(rng.integers(0, depth + 1))
        path = tuple(int(x) for x in rng.integers(0, branching, size=d))
        parts = [tokens(root, path[:k]) for k in range(d + 1)]
        full = np.concatenate(parts)
        length = int(rng.integers(min_len, max_len + 1))
        if length <= full.size:
            prompt = full[:length]
        else:
            extra = rng.integers(0, vocabulary, size=length - full.size, dtype=np.int64).astype(np.int32)
            prompt = np.concatenate([full, extra])
        new = int(rng.integers(min_new, max_new + 1))
        out.append(PrefixTreeRequest(root, path, prompt.astype(np.int32), new))
    return out
