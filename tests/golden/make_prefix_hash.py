"""Write tests/golden/prefix_hash.json: block keys computed by the reference itself.

Run where the reference sources are present:

    HELIOS_REFERENCE_SRC=<reference>/src python tests/golden/make_prefix_hash.py

It imports ``helios.runtime.prefix_cache.build_token_blocks`` unchanged and records, for
seeded prompts (lengths 0 to 700, ids from 0 to 2^31 - 1, block sizes 1, 7 and 256), every
block's hex key and parent key. The tests read the file; nothing at test time imports the
reference.
"""

from __future__ import annotations

import json
import os
import random
import sys
from pathlib import Path


def prompts() -> list[tuple[list[int], int]]:
    rng = random.Random(11)
    cases = [([], 4), ([0], 1), ([0, 1, 2, 3, 4, 5, 6], 7), ([2 ** 31 - 1] * 9, 4)]
    for block_size, n in ((1, 40), (7, 300), (256, 700), (256, 512)):
        cases.append(([rng.randrange(151936) for _ in range(n)], block_size))
    cases.append(([rng.choice([0, 9, 10, 99, 100, 151935, 2 ** 31 - 1]) for _ in range(33)], 5))
    return cases


def main() -> None:
    sys.path.insert(0, os.environ["HELIOS_REFERENCE_SRC"])
    from helios.runtime.prefix_cache import build_token_blocks

    out = []
    for tokens, block_size in prompts():
        blocks = build_token_blocks(tokens, block_size)
        out.append({"tokens": tokens, "block_size": block_size,
                    "hashes": [b.hash for b in blocks], "parents": [b.parent_hash for b in blocks]})
    path = Path(__file__).with_name("prefix_hash.json")
    path.write_text(json.dumps(out, separators=(",", ":")))
    print(f"wrote {path} ({len(out)} prompts)")


if __name__ == "__main__":
    main()
