"""Qwen3 decoder over the paged caches, running the B200 kernels.

Module tree, parameter names and construction order are the reference's
(src/helios/runtime/qwen3/model.py:13-30, layers.py:13-232): ``token_embedding``,
``blocks.{i}.attention.{query,key,value,output,q_norm,k_norm}``,
``blocks.{i}.feed_forward.{gate,up,down}``, ``blocks.{i}.{input_norm,post_attention_norm}``,
``final_norm``, ``output`` tied to the embedding, fp32 norm scales and fp32
``cos``/``sin`` buffers. So ``load_state_dict`` of reference weights works and
``torch.manual_seed(s); Qwen3Model(config)`` draws the same random weights.

The forward is the packed mixed-batch path of ``Qwen3Model._forward_packed``
(model.py:92-110), restated for one flattened token dimension:

    x = embed(ids)                                       kernel: embed
    n = rmsnorm(x, input_norm_0)                         kernel: rmsnorm
    per layer:
      qkv = n @ [Wq; Wk; Wv]^T                           cuBLAS GEMM (one, fused weights)
      q = attend(norm+rope(q), append(norm+rope(k), v))  kernels b + c
      h, n2 = x + q @ Wo^T, rmsnorm(.)                   GEMM + kernel: add_rmsnorm
      m = silu(n2 @ Wg^T) * (n2 @ Wu^T) @ Wd^T           tcgen05 gate|up GEMM with SwiGLU epilogue + GEMM
      x, n = h + m, rmsnorm(., next norm)                kernel: add_rmsnorm
    logits = n[logit rows] @ E^T                         GEMM

Every bf16 rounding point of the reference is kept (projection outputs,
residual sums, silu output, gated product, norms). Decode-only and uniform
prefill ticks (``PagedBatchCache`` + ``prepare(tokens)``, model.py:32-90,
:133-169) use the same path with one logit row per sequence.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
import torch.nn.functional as F
from torch import nn

from helios_b200 import ops
from helios_b200.config import Qwen3Config
from helios_b200.paged_cache import PackedBatchCache, PagedBatchCache


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float) -> None:
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        flat = x.reshape(-1, x.shape[-1])
        return ops.rmsnorm(flat.contiguous(), self.scale, self.eps).view(x.shape)


def rope_parameters(config: Qwen3Config) -> tuple[torch.Tensor, torch.Tensor]:
    """Same tables as layers.py:43-51: angles = pos * theta^(-2i/d), duplicated halves.
    Always computed on the CPU, as the reference builds them before moving the model, so
    the fp32 tables are the reference's bit for bit whatever device the model lives on."""
    cpu = torch.device("cpu")
    inverse = 1.0 / (config.rope_base ** (torch.arange(0, config.head_dim, 2, dtype=torch.float32, device=cpu)
                                          / config.head_dim))
    angles = torch.arange(config.context_length, dtype=torch.float32, device=cpu).unsqueeze(1) * inverse.unsqueeze(0)
    angles = torch.cat((angles, angles), dim=1)
    return torch.cos(angles), torch.sin(angles)


# Token rows from which the fused tcgen05 gate|up + SwiGLU kernel is used. Measured at the
# Qwen3-4B shape (gate|up weights cycled beyond L2): it matches cuBLAS + the SwiGLU kernel at
# 128 and 1280 rows, trails it between (39 vs 30 us at 256, 87 vs 82 us at 1024) and leads
# from 1536 rows (120 vs 126 us; 156 vs 182 us at the 2080-row tick).
FUSED_GATE_UP_MIN_ROWS = 1280
# Decode-tick projections (a few to 256 token rows) stay on cuBLAS: measured at the Qwen3-4B
# shapes with 128 rows, q|k|v 8.9 us, output 8.5, gate|up 22.4, down 16.4 (56 us per layer,
# 0.55 of the copy peak over the 202 MB of weights), ahead of a stream-K weight-streaming tcgen05
# GEMM written for them (41, 57, 45, 61 us): splitting 2560-row outputs over 148 SMs leaves
# each output tile in ~8 fp32 parts whose in-order reduction is latency-bound.


class _Fused:
    """Concatenation of several Linear weights along the output dimension, rebuilt
    when any of them is replaced or modified in place (e.g. by load_state_dict)."""

    def __init__(self, *linears: nn.Linear) -> None:
        self.linears = linears
        self.key = None
        self.weight: torch.Tensor | None = None

    def _key(self):
        return tuple((l.weight.data_ptr(), l.weight._version, l.weight.device) for l in self.linears)

    def get(self) -> torch.Tensor:
        if self._key() != self.key:
            # Normal (not inference-mode) tensors, so the weights stay loadable afterwards.
            with torch.inference_mode(False), torch.no_grad():
                fused = torch.cat([l.weight for l in self.linears], dim=0).contiguous()
                # Point the Linear weights at slices of the fused copy: no duplicate storage.
                start = 0
                for l in self.linears:
                    n = l.weight.shape[0]
                    l.weight = nn.Parameter(fused[start:start + n], requires_grad=False)
                    start += n
            self.weight = fused
            self.key = self._key()
        return self.weight


class FeedForward(nn.Module):
    def __init__(self, config: Qwen3Config) -> None:
        super().__init__()
        self.gate = nn.Linear(config.hidden_size, config.hidden_dim, bias=False, dtype=config.dtype)
        self.up = nn.Linear(config.hidden_size, config.hidden_dim, bias=False, dtype=config.dtype)
        self.down = nn.Linear(config.hidden_dim, config.hidden_size, bias=False, dtype=config.dtype)
        self._gate_up = _Fused(self.gate, self.up)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """``x [T, hidden]`` -> ``[T, hidden]``: gate|up projection + SwiGLU, then the down GEMM.
        From FUSED_GATE_UP_MIN_ROWS rows the gate|up GEMM runs on this library's tcgen05 kernel
        with SwiGLU in its epilogue; fewer rows (mostly padding in its 128-row tiles) take
        cuBLAS and the SwiGLU kernel. Both keep the reference's rounding points."""
        inter = self.gate.out_features
        if x.shape[0] >= FUSED_GATE_UP_MIN_ROWS and x.shape[1] % 64 == 0 and inter % 128 == 0:
            act = ops.gemm_swiglu(x.contiguous(), self._gate_up.get())
        else:
            gate_up = F.linear(x, self._gate_up.get())
            act = torch.empty((x.shape[0], inter), dtype=x.dtype, device=x.device)
            ops.swiglu(gate_up, act)
        return F.linear(act, self.down.weight)


class GroupedQueryAttention(nn.Module):
    def __init__(self, config: Qwen3Config) -> None:
        super().__init__()
        if config.n_heads % config.n_kv_heads:
            raise ValueError("The number of Q heads must be divisible by the number of KV heads.")
        self.n_heads = config.n_heads
        self.n_kv_heads = config.n_kv_heads
        self.group_size = config.n_heads // config.n_kv_heads
        self.head_dim = config.head_dim
        self.query = nn.Linear(config.hidden_size, config.n_heads * config.head_dim, bias=False, dtype=config.dtype)
        self.key = nn.Linear(config.hidden_size, config.n_kv_heads * config.head_dim, bias=False, dtype=config.dtype)
        self.value = nn.Linear(config.hidden_size, config.n_kv_heads * config.head_dim, bias=False, dtype=config.dtype)
        self.output = nn.Linear(config.n_heads * config.head_dim, config.hidden_size, bias=False, dtype=config.dtype)
        self.q_norm = RMSNorm(config.head_dim, config.rms_norm_eps)
        self.k_norm = RMSNorm(config.head_dim, config.rms_norm_eps)
        self._qkv = _Fused(self.query, self.key, self.value)

    def forward(self, x: torch.Tensor, cache: PagedBatchCache, layer_index: int, cos: torch.Tensor,
                sin: torch.Tensor) -> torch.Tensor:
        """``x [T, hidden]`` (already input-normed) -> attention block output ``[T, hidden]``:
        one cuBLAS GEMM for q|k|v, kernel (b) (norm, RoPE, KV append), kernel (c), o-proj."""
        qkv = F.linear(x, self._qkv.get())
        context = cache.attend_fused(layer_index, qkv, self.q_norm.scale, self.k_norm.scale, self.q_norm.eps,
                                     cos, sin)
        return F.linear(context.view(x.shape[0], -1), self.output.weight)


class TransformerBlock(nn.Module):
    def __init__(self, config: Qwen3Config) -> None:
        super().__init__()
        self.attention = GroupedQueryAttention(config)
        self.feed_forward = FeedForward(config)
        self.input_norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_norm = RMSNorm(config.hidden_size, config.rms_norm_eps)


class Qwen3Model(nn.Module):
    def __init__(self, config: Qwen3Config) -> None:
        super().__init__()
        self.config = config
        self.token_embedding = nn.Embedding(config.vocab_size, config.hidden_size, dtype=config.dtype)
        self.blocks = nn.ModuleList(TransformerBlock(config) for _ in range(config.n_layers))
        self.final_norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.output = nn.Linear(config.hidden_size, config.vocab_size, bias=False, dtype=config.dtype)
        self.output.weight = self.token_embedding.weight
        cos, sin = rope_parameters(config)
        device = self.token_embedding.weight.device  # the device the module is being built on
        self.register_buffer("cos", cos.to(device), persistent=False)
        self.register_buffer("sin", sin.to(device), persistent=False)
        self._graphs = None  # TickGraphs once enable_cuda_graphs() is called

    @classmethod
    def from_state_dict(cls, config: Qwen3Config, state_dict: dict[str, torch.Tensor],
                        device: torch.device | str) -> "Qwen3Model":
        """A model on ``device`` holding ``state_dict`` (reference names, e.g. a reference
        ``Qwen3Model.state_dict()`` or a loaded checkpoint), without drawing random weights
        first: the modules are built on the meta device, materialised on ``device`` and
        filled. Every parameter must be in ``state_dict``."""
        with torch.device("meta"):
            model = cls(config)
        model = model.to_empty(device=device)
        model.output.weight = model.token_embedding.weight  # materialising unties them
        cos, sin = rope_parameters(config)
        model.cos.copy_(cos)
        model.sin.copy_(sin)
        missing, unexpected = model.load_state_dict(state_dict, strict=False)
        missing = [k for k in missing if k not in ("output.weight",)]
        if missing or unexpected:
            raise ValueError(f"state dict does not match the model: missing {missing}, unexpected {unexpected}")
        return model.eval()

    def enable_cuda_graphs(self, max_graphs: int = 4) -> None:
        """Replay the device half of packed ticks from CUDA graphs (see helios_b200.graphs).
        Logits are identical to eager ticks; the returned logits tensor is reused by the
        next tick of the same shape."""
        from helios_b200.graphs import TickGraphs

        self._graphs = TickGraphs(self, max_graphs)

    def forward(self, input_ids: torch.Tensor, cache: PagedBatchCache | None = None,
                position_ids: torch.Tensor | None = None,
                cache_slots: Sequence[int] | torch.Tensor | None = None) -> torch.Tensor:
        """Reference signature (model.py:32-90). Packed caches return ``[logit rows, V]``;
        uniform paged batches return the last position of each row, ``[B, 1, V]``.
        Positions always come from the paged cache (``position_ids`` is accepted for
        signature compatibility; the reference derives the same values)."""
        out = self._run(input_ids, cache, cache_slots, greedy=False)
        return out if isinstance(cache, PackedBatchCache) else out.view(cache.batch_size, 1, -1)

    def greedy_ids(self, input_ids: torch.Tensor, cache: PagedBatchCache,
                   cache_slots: Sequence[int] | torch.Tensor | None = None) -> torch.Tensor:
        """Temperature-0 token ids of the rows ``forward`` returns logits for (int64: ``[logit rows]``
        for packed caches, ``[B]`` for uniform paged batches): the argmax of those bf16 logits with
        ties to the lowest id (decode.py:458-460), from the lm_head GEMM with the argmax in its
        epilogue, so the logits are never written (hb_lm_head_argmax)."""
        return self._run(input_ids, cache, cache_slots, greedy=True)

    def _run(self, input_ids: torch.Tensor, cache, cache_slots, *, greedy: bool) -> torch.Tensor:
        if isinstance(cache, PackedBatchCache):
            if input_ids.shape != (1, sum(cache.counts)):
                raise ValueError("Packed input does not match query lengths.")
            out = self._device_half(input_ids, cache, greedy)
            cache.advance_packed()
            return out
        if not isinstance(cache, PagedBatchCache):
            raise TypeError("The B200 model runs over paged KV caches (PagedBatchCache / PackedBatchCache).")
        if cache_slots is not None:
            cache.slot_ids(cache_slots)
        tokens = input_ids.shape[1]
        if input_ids.shape[0] != cache.batch_size:
            raise ValueError("Paged input rows must match the paged batch.")
        if max(c.length + tokens for c in cache.caches) > self.config.context_length:
            raise ValueError(f"Qwen3-4B supports at most {self.config.context_length:,} tokens per request.")
        # prepare(tokens) packed one logit row per sequence: its last position.
        out = self._device_half(input_ids, cache, greedy)
        cache.advance(tokens, slots=cache_slots)
        return out

    def _device_half(self, input_ids: torch.Tensor, cache: PagedBatchCache, greedy: bool) -> torch.Tensor:
        if self._graphs is not None and input_ids.is_cuda:
            return self._graphs.run(input_ids, cache, greedy=greedy)
        return self._packed_logits(input_ids.reshape(-1), cache, greedy=greedy)

    def _packed_logits(self, ids: torch.Tensor, cache: PagedBatchCache, *, greedy: bool = False) -> torch.Tensor:
        """Device half of a prepared tick: logits of the cache's logit rows (or, ``greedy``, their
        argmax ids). It makes no host synchronisation, so it can be captured into a CUDA graph."""
        _, normed = self._layers(ids, cache)
        rows = normed.index_select(0, cache.logit_rows)
        if greedy:
            return ops.lm_head_argmax(rows, self.output.weight)
        return F.linear(rows, self.output.weight)

    def _layers(self, ids: torch.Tensor, cache: PagedBatchCache) -> tuple[torch.Tensor, torch.Tensor]:
        """Run every block; returns (residual stream, final-normed stream) ``[T, hidden]``."""
        if ids.dtype != torch.long:
            ids = ids.long()
        ids = ids.contiguous()
        tokens, hidden = ids.numel(), self.config.hidden_size
        eps = self.config.rms_norm_eps
        dev, dt = self.token_embedding.weight.device, self.config.dtype
        x = ops.embedding(ids, self.token_embedding.weight, torch.empty((tokens, hidden), dtype=dt, device=dev))
        normed = ops.rmsnorm(x, self.blocks[0].input_norm.scale, eps)
        h = torch.empty_like(x)
        normed2 = torch.empty_like(x)
        for index, block in enumerate(self.blocks):
            attn = block.attention(normed, cache, index, self.cos, self.sin)
            ops.add_rmsnorm(x, attn, block.post_attention_norm.scale, eps, h, normed2)
            mlp = block.feed_forward(normed2)
            nxt = self.blocks[index + 1].input_norm.scale if index + 1 < len(self.blocks) else self.final_norm.scale
            ops.add_rmsnorm(h, mlp, nxt, eps, x, normed)
        return x, normed
