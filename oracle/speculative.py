"""Speculative verification oracle.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates the acceptance loop of ``Engine._execute_batch``
(src/helios/runtime/engine.py:488-520): a decoding row's chunk is ``[pending, d1, ..., dk]``
with one logit row per chunk token; ``verified`` holds the greedy id of every logit row
(``logits.argmax(dim=-1)``, :488-489); the row accepts the longest prefix of its drafts
``d1..dk`` equal to its predictions, truncates its cache to ``length + 1 + accepted``
(:515) and emits ``predictions[: accepted + 1]`` (:517). A row with one logit row emits
its (sampled) head.
"""

from __future__ import annotations

from collections.abc import Sequence


def accept(chunks: Sequence[Sequence[int]], logit_counts: Sequence[int],
           predictions: Sequence[int]) -> tuple[list[int], list[list[int]]]:
    """(accepted per row, tokens emitted per row) for greedy ``predictions`` of every logit row."""
    accepted, emitted, start = [], [], 0
    for chunk, lc in zip(chunks, logit_counts, strict=True):
        row_pred = list(predictions[start: start + lc])
        if lc > 1:
            n = 0
            for proposal, prediction in zip(chunk[1:], row_pred):
                if proposal != prediction:
                    break
                n += 1
            accepted.append(n)
            emitted.append(row_pred[: n + 1])
        else:
            accepted.append(0)
            emitted.append(row_pred[:1])
        start += lc
    return accepted, emitted
