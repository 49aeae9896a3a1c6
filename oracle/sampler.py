"""Sampling oracle: greedy, temperature and top-p (nucleus) selection.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates ``Decoder._sample`` (src/helios/runtime/qwen3/decode.py:457-473) and
its batched use in ``Engine._execute_batch`` (src/helios/runtime/engine.py:470-492):

  * temperature 0 -> ``argmax`` (first index among equal maxima);
  * otherwise ``p = softmax(logits / T)``; when ``top_p < 1`` the probabilities
    are sorted in descending order and token j of that order is removed when
    the inclusive cumulative sum of the tokens *before* it exceeds ``top_p``
    (``remove`` shifted right by one, first token always kept, :467-469); the
    survivors are renormalised and one is drawn.

The reference draws with ``torch.multinomial`` whose random stream cannot be
reproduced, so the draw is restated for a caller-supplied uniform ``u`` in
[0, 1): the kept tokens are visited in ascending token index and the first
whose running mass exceeds ``u * kept_mass`` is returned. The distribution is
the reference's; the deterministic rule is what the CUDA sampler implements.
Arithmetic here is fp32 from the (bf16) logits; ties in probability are ordered
by ascending token index.
"""

from __future__ import annotations

import torch


def greedy(logits: torch.Tensor) -> torch.Tensor:
    return torch.argmax(logits.float(), dim=-1)


def probabilities(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    scaled = logits.float() / temperature
    return torch.softmax(scaled, dim=-1)


def keep_mask(logits: torch.Tensor, temperature: float, top_p: float) -> torch.Tensor:
    """Boolean ``[rows, V]`` of tokens that survive the top-p cut (decode.py:464-470)."""
    probs = probabilities(logits, temperature)
    if top_p >= 1.0:
        return torch.ones_like(probs, dtype=torch.bool)
    # Stable order: descending probability, ascending index within ties.
    sorted_probs, order = torch.sort(probs, dim=-1, descending=True, stable=True)
    before = torch.cumsum(sorted_probs.double(), dim=-1) - sorted_probs.double()
    keep_sorted = before <= top_p
    keep_sorted[..., 0] = True
    mask = torch.zeros_like(keep_sorted)
    mask.scatter_(-1, order, keep_sorted)
    return mask


def sample(logits: torch.Tensor, temperature: float, top_p: float, uniforms: torch.Tensor) -> torch.Tensor:
    """Deterministic draw for each row given ``uniforms[rows]`` in [0, 1)."""
    if temperature == 0:
        return greedy(logits)
    probs = probabilities(logits, temperature).double()
    kept = keep_mask(logits, temperature, top_p)
    probs = probs * kept
    out = torch.empty(probs.shape[0], dtype=torch.long)
    for row in range(probs.shape[0]):
        running = torch.cumsum(probs[row], dim=0)
        target = float(uniforms[row]) * float(running[-1])
        hit = torch.nonzero((running > target) & kept[row], as_tuple=False)
        out[row] = int(hit[0]) if len(hit) else int(torch.nonzero(kept[row])[-1])
    return out


def boundary_distance(logits: torch.Tensor, temperature: float, uniforms: torch.Tensor, top_p: float) -> torch.Tensor:
    """Distance of ``u * kept_mass`` from the nearest cumulative-mass edge, per row.

    Two correct implementations that sum in different orders may pick adjacent
    tokens only when this distance is within float rounding; tests use it to
    tell rounding from disagreement.
    """
    probs = probabilities(logits, temperature).double() * keep_mask(logits, temperature, top_p)
    out = torch.empty(probs.shape[0], dtype=torch.float64)
    for row in range(probs.shape[0]):
        running = torch.cumsum(probs[row], dim=0)
        target = float(uniforms[row]) * float(running[-1])
        out[row] = torch.min(torch.abs(running - target))
    return out
