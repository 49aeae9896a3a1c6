"""Qwen3 weights and packed forward oracle.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

  * ``OracleConfig`` mirrors the fields of ``Qwen3Config``
    (src/helios/runtime/qwen3/config.py:8-20).
  * ``build_state_dict`` creates the reference's random-init weights: the same
    PyTorch modules (``nn.Embedding``, bias-free ``nn.Linear``) created in the
    order ``Qwen3Model.__init__`` creates them (model.py:14-27, layers.py:76-111,
    :195-200, :13-24), under ``torch.manual_seed(seed)``; norm scales are fp32
    ones (layers.py:34); the output projection is tied to the embedding
    (model.py:27). State-dict names are the reference's.
  * ``OracleModel.forward_packed`` restates ``Qwen3Model._forward_packed``
    (model.py:92-110) with ``TransformerBlock.forward`` (layers.py:202-232),
    ``GroupedQueryAttention.forward`` (layers.py:113-164), ``FeedForward``
    (layers.py:26-27) and the packed paged cache (paged_cache.py:501-546). Every
    bf16 rounding point of the reference is kept: projections, ``silu`` output,
    the gated product and both residual adds round to the model dtype.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from oracle.attention import paged_attention, write_pool
from oracle.metadata import pack_tick
from oracle.numerics import apply_rope, rms_norm, rope_tables


@dataclass(frozen=True)
class OracleConfig:
    vocab_size: int = 151_936
    context_length: int = 40_960
    hidden_size: int = 2_560
    n_heads: int = 32
    n_layers: int = 36
    hidden_dim: int = 9_728
    head_dim: int = 128
    n_kv_heads: int = 8
    rope_base: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    dtype: torch.dtype = torch.bfloat16


def build_state_dict(config: OracleConfig, seed: int, *, layers: int | None = None,
                     rng_checkpoints: list[torch.Tensor] | None = None,
                     threads: int = 1) -> dict[str, torch.Tensor]:
    """Reference random-init weights for ``torch.manual_seed(seed)``.

    ``layers`` truncates the stack (the first ``layers`` blocks are identical to
    the full model's, since blocks are created in order).

    The reference draws every tensor from the one CPU generator in creation order,
    which takes minutes at the Qwen3-4B shape. With ``rng_checkpoints`` (the generator
    state before the embedding and before each block, from ``rng_checkpoints``) the
    embedding and the blocks are drawn from their own generators, set to those states,
    on ``threads`` threads: the same draws, so the same bits.
    """
    c = config
    n = c.n_layers if layers is None else layers
    if rng_checkpoints is not None:
        return _build_from_checkpoints(c, n, rng_checkpoints, threads)
    torch.manual_seed(seed)
    sd: dict[str, torch.Tensor] = {}
    sd["token_embedding.weight"] = nn.Embedding(c.vocab_size, c.hidden_size, dtype=c.dtype).weight.data
    for i in range(n):
        p = f"blocks.{i}."
        sd[p + "attention.query.weight"] = nn.Linear(c.hidden_size, c.n_heads * c.head_dim, bias=False, dtype=c.dtype).weight.data
        sd[p + "attention.key.weight"] = nn.Linear(c.hidden_size, c.n_kv_heads * c.head_dim, bias=False, dtype=c.dtype).weight.data
        sd[p + "attention.value.weight"] = nn.Linear(c.hidden_size, c.n_kv_heads * c.head_dim, bias=False, dtype=c.dtype).weight.data
        sd[p + "attention.output.weight"] = nn.Linear(c.n_heads * c.head_dim, c.hidden_size, bias=False, dtype=c.dtype).weight.data
        sd[p + "attention.q_norm.scale"] = torch.ones(c.head_dim)
        sd[p + "attention.k_norm.scale"] = torch.ones(c.head_dim)
        sd[p + "feed_forward.gate.weight"] = nn.Linear(c.hidden_size, c.hidden_dim, bias=False, dtype=c.dtype).weight.data
        sd[p + "feed_forward.up.weight"] = nn.Linear(c.hidden_size, c.hidden_dim, bias=False, dtype=c.dtype).weight.data
        sd[p + "feed_forward.down.weight"] = nn.Linear(c.hidden_dim, c.hidden_size, bias=False, dtype=c.dtype).weight.data
        sd[p + "input_norm.scale"] = torch.ones(c.hidden_size)
        sd[p + "post_attention_norm.scale"] = torch.ones(c.hidden_size)
    sd["final_norm.scale"] = torch.ones(c.hidden_size)
    sd["output.weight"] = sd["token_embedding.weight"]
    return sd


def _linear_weight(out_features: int, in_features: int, dtype: torch.dtype, generator: torch.Generator) -> torch.Tensor:
    """``nn.Linear(in, out, bias=False).weight`` drawn from ``generator`` (Linear.reset_parameters)."""
    w = torch.empty((out_features, in_features), dtype=dtype)
    nn.init.kaiming_uniform_(w, a=math.sqrt(5), generator=generator)
    return w


def _block_state(c: OracleConfig, i: int, generator: torch.Generator) -> dict[str, torch.Tensor]:
    p = f"blocks.{i}."
    qd, kvd = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
    return {
        p + "attention.query.weight": _linear_weight(qd, c.hidden_size, c.dtype, generator),
        p + "attention.key.weight": _linear_weight(kvd, c.hidden_size, c.dtype, generator),
        p + "attention.value.weight": _linear_weight(kvd, c.hidden_size, c.dtype, generator),
        p + "attention.output.weight": _linear_weight(c.hidden_size, qd, c.dtype, generator),
        p + "attention.q_norm.scale": torch.ones(c.head_dim),
        p + "attention.k_norm.scale": torch.ones(c.head_dim),
        p + "feed_forward.gate.weight": _linear_weight(c.hidden_dim, c.hidden_size, c.dtype, generator),
        p + "feed_forward.up.weight": _linear_weight(c.hidden_dim, c.hidden_size, c.dtype, generator),
        p + "feed_forward.down.weight": _linear_weight(c.hidden_size, c.hidden_dim, c.dtype, generator),
        p + "input_norm.scale": torch.ones(c.hidden_size),
        p + "post_attention_norm.scale": torch.ones(c.hidden_size),
    }


def rng_checkpoints(config: OracleConfig, seed: int) -> list[torch.Tensor]:
    """CPU generator states before the embedding and before each block of the
    reference's seed-``seed`` initialisation (one serial pass over every draw)."""
    torch.manual_seed(seed)
    states = [torch.get_rng_state()]
    c = config
    nn.Embedding(c.vocab_size, c.hidden_size, dtype=c.dtype)
    generator = torch.default_generator
    for i in range(c.n_layers):
        states.append(torch.get_rng_state())
        _block_state(c, i, generator)
    return states


def _build_from_checkpoints(c: OracleConfig, n: int, states: list[torch.Tensor], threads: int) -> dict[str, torch.Tensor]:
    from concurrent.futures import ThreadPoolExecutor

    if len(states) < n + 1:
        raise ValueError("Need a generator state for the embedding and for every block.")

    def embedding():
        g = torch.Generator()
        g.set_state(states[0])
        w = torch.empty((c.vocab_size, c.hidden_size), dtype=c.dtype)
        nn.init.normal_(w, generator=g)
        return {"token_embedding.weight": w}

    def block(i):
        g = torch.Generator()
        g.set_state(states[i + 1])
        return _block_state(c, i, g)

    with ThreadPoolExecutor(max(1, threads)) as pool:
        parts = list(pool.map(lambda job: job(), [embedding] + [lambda i=i: block(i) for i in range(n)]))
    sd: dict[str, torch.Tensor] = {}
    for part in parts:
        sd.update(part)
    sd["final_norm.scale"] = torch.ones(c.hidden_size)
    sd["output.weight"] = sd["token_embedding.weight"]
    return sd


def new_pools(config: OracleConfig, num_pages: int, page_size: int = 256, layers: int | None = None):
    """Per-layer K and V pools ``[P, page, Hkv, d]`` (paged_cache.py:47-55), zero-filled."""
    n = config.n_layers if layers is None else layers
    shape = (num_pages, page_size, config.n_kv_heads, config.head_dim)
    return [torch.zeros(shape, dtype=config.dtype) for _ in range(n)], [torch.zeros(shape, dtype=config.dtype) for _ in range(n)]


class OracleModel:
    def __init__(self, config: OracleConfig, state_dict: dict[str, torch.Tensor], *, layers: int | None = None):
        self.config = config
        self.sd = state_dict
        self.layers = config.n_layers if layers is None else layers
        self.cos, self.sin = rope_tables(config.head_dim, config.context_length, config.rope_base)

    def _block(self, i: int, x: torch.Tensor, key_pool, value_pool, meta: dict) -> torch.Tensor:
        c, sd, p = self.config, self.sd, f"blocks.{i}."
        tokens = x.shape[0]
        h = rms_norm(x, sd[p + "input_norm.scale"], c.rms_norm_eps)
        q = F.linear(h, sd[p + "attention.query.weight"]).view(tokens, c.n_heads, c.head_dim).transpose(0, 1)
        k = F.linear(h, sd[p + "attention.key.weight"]).view(tokens, c.n_kv_heads, c.head_dim).transpose(0, 1)
        v = F.linear(h, sd[p + "attention.value.weight"]).view(tokens, c.n_kv_heads, c.head_dim)
        positions = torch.as_tensor(meta["positions"], dtype=torch.long)
        q = apply_rope(rms_norm(q, sd[p + "attention.q_norm.scale"], c.rms_norm_eps), self.cos, self.sin, positions)
        k = apply_rope(rms_norm(k, sd[p + "attention.k_norm.scale"], c.rms_norm_eps), self.cos, self.sin, positions)
        write_pool(key_pool, meta["write_slots"], k.transpose(0, 1))
        write_pool(value_pool, meta["write_slots"], v)
        context = paged_attention(
            q.transpose(0, 1).contiguous(), key_pool, value_pool,
            meta["block_table"], meta["cu_seq_q"], meta["seqused_k"],
        )
        x = x + F.linear(context.reshape(tokens, -1), sd[p + "attention.output.weight"])
        h = rms_norm(x, sd[p + "post_attention_norm.scale"], c.rms_norm_eps)
        gated = F.silu(F.linear(h, sd[p + "feed_forward.gate.weight"])) * F.linear(h, sd[p + "feed_forward.up.weight"])
        return x + F.linear(gated, sd[p + "feed_forward.down.weight"])

    def forward_packed(self, token_ids, key_pools, value_pools, meta: dict) -> torch.Tensor:
        """Logits ``[len(logit_indices), vocab]`` in the model dtype."""
        ids = torch.as_tensor(list(token_ids), dtype=torch.long)
        x = self.sd["token_embedding.weight"][ids]
        for i in range(self.layers):
            x = self._block(i, x, key_pools[i], value_pools[i], meta)
        x = x[torch.as_tensor(meta["logit_indices"], dtype=torch.long)]
        x = rms_norm(x, self.sd["final_norm.scale"], self.config.rms_norm_eps)
        return F.linear(x, self.sd["output.weight"])


class OracleRequests:
    """Minimal page bookkeeping for driving ``OracleModel`` tick by tick.

    Pages are handed out LIFO from ``range(P-1, -1, -1)`` as ``KVPagePool``
    does (paged_cache.py:56, :76-86).
    """

    def __init__(self, num_pages: int, page_size: int = 256):
        self.page_size = page_size
        self.free = list(range(num_pages - 1, -1, -1))
        self.lengths: list[int] = []
        self.capacities: list[int] = []
        self.tables: list[list[int]] = []

    def add(self, capacity: int) -> int:
        self.lengths.append(0)
        self.capacities.append(capacity)
        self.tables.append([])
        return len(self.lengths) - 1

    def tick(self, rows, counts, logit_counts=None) -> dict:
        for row, count in zip(rows, counts):
            need = -(-(self.lengths[row] + count) // self.page_size) - len(self.tables[row])
            for _ in range(max(0, need)):
                self.tables[row].append(self.free.pop())
        return pack_tick(
            [self.lengths[r] for r in rows], counts, [self.tables[r] for r in rows],
            [self.capacities[r] for r in rows], logit_counts=logit_counts, page_size=self.page_size,
        )

    def advance(self, rows, counts) -> None:
        for row, count in zip(rows, counts):
            self.lengths[row] += count
