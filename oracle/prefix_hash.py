"""Prefix-cache block keys and longest-prefix lookup: TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates, with the standard library, how the reference keys its prefix cache:

* ``hash_token_blocks`` (src/helios/runtime/prefix_cache.py:86-106): a prompt is cut into
  blocks of ``block_size`` tokens (``split_token_stream``, :76-83; the last block may be
  partial); block i's key is SHA-256 over the previous block's raw digest (nothing for
  block 0) followed by the block's tokens as compact JSON, ``"[t0,t1,...]"``.
* the probe loop of ``PrefixCache.longest_prefix`` (:208-222): walk the prompt's blocks in
  order, stop at the first partial block or the first key that is not stored.

Pinned against keys the reference itself computed (``tests/golden/prefix_hash.json``,
written by ``tests/golden/make_prefix_hash.py``).
"""

from __future__ import annotations

import hashlib
import json
from collections.abc import Mapping, Sequence


def block_keys(tokens: Sequence[int], block_size: int) -> list[bytes]:
    """Raw 32-byte keys of every block of ``tokens``, partial last block included."""
    if block_size < 1:
        raise ValueError("block_size must be at least 1.")
    keys, parent = [], b""
    for start in range(0, len(tokens), block_size):
        block = tuple(int(t) for t in tokens[start:start + block_size])
        payload = json.dumps(block, separators=(",", ":")).encode("ascii")
        parent = hashlib.sha256(parent + payload).digest()
        keys.append(parent)
    return keys


def longest_prefix(tokens: Sequence[int], block_size: int, stored: Mapping[bytes, int]) -> list[int]:
    """Values of the leading full blocks whose keys are stored, up to the first that is not."""
    out = []
    for index, key in enumerate(block_keys(tokens, block_size)):
        if len(tokens[index * block_size:(index + 1) * block_size]) != block_size or key not in stored:
            break
        out.append(stored[key])
    return out
