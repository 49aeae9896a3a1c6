"""Device-resident prefix index: block keys on the GPU and the longest-prefix walk.

Keys must equal the reference's ``build_token_blocks`` hashes (prefix_cache.py:86-110)
bit for bit: the golden file holds keys the reference computed, and random prompts are
checked against the oracle's hashlib restatement. Lookups must match the oracle's walk of
``PrefixCache.longest_prefix`` (:208-222) over the same stored keys, through insertions and
removals.
"""

import json
import random

import pytest
import torch

from helios_b200 import _native
from helios_b200.prefix_index import DevicePrefixIndex, hash_token_blocks
from oracle.prefix_hash import block_keys, longest_prefix

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def test_keys_match_the_reference_golden_keys(golden_dir):
    cases = json.loads((golden_dir / "prefix_hash.json").read_text())
    for case in cases:
        got = hash_token_blocks([case["tokens"]], case["block_size"], DEV)[0]
        assert got == case["hashes"], case["block_size"]
        assert [""] + got[:-1] == case["parents"] if got else not case["parents"]
    assert _native.device_status() == 0


@pytest.mark.parametrize("block_size", [1, 7, 256])
def test_keys_of_a_batch_match_the_oracle(block_size):
    rng = random.Random(block_size)
    values = [0, 1, 9, 10, 151935, 2 ** 31 - 1]
    prompts = []
    for i in range(300):  # more prompts than one CTA's threads
        n = rng.randrange(0, 40 if block_size == 1 else 900)
        prompts.append([rng.choice(values) if rng.random() < 0.1 else rng.randrange(151936) for _ in range(n)])
    got = hash_token_blocks(prompts, block_size, DEV)
    for tokens, keys in zip(prompts, got):
        assert keys == [k.hex() for k in block_keys(tokens, block_size)]
    assert _native.device_status() == 0


def test_lookup_walks_stored_blocks_like_longest_prefix():
    rng = random.Random(3)
    bs = 16
    shared = [rng.randrange(151936) for _ in range(5 * bs)]
    a = shared + [rng.randrange(151936) for _ in range(2 * bs + 3)]        # 7 full blocks + partial
    b = shared[:3 * bs] + [rng.randrange(151936) for _ in range(4 * bs)]   # diverges at block 3
    c = [rng.randrange(151936) for _ in range(6 * bs)]                      # nothing stored
    d = shared[:bs - 1]                                                      # partial only
    e = a[:4 * bs]                                                           # exact 4-block prefix of a
    prompts = [a, b, c, d, e, []]
    index = DevicePrefixIndex(capacity=64, block_size=bs, device=DEV)
    stored: dict[bytes, int] = {}

    def store(tokens, blocks, base):
        keys = [k for k in block_keys(tokens, bs)[:blocks] if k not in stored]
        vals = [base + i for i in range(len(keys))]
        index.add([k.hex() for k in keys], vals)
        stored.update(zip(keys, vals))

    def check():
        got = index.lookup(prompts)
        for tokens, (keys, vals) in zip(prompts, got):
            want = longest_prefix(tokens, bs, stored)
            assert vals == want
            assert keys == [k.hex() for k in block_keys(tokens, bs)[:len(want)]]
        return [len(v) for _, v in got]

    store(a, 7, 100)
    store(b, 5, 200)
    assert check() == [7, 5, 0, 0, 4, 0]
    removed = block_keys(a, bs)[2]  # evict a's third block: a and e stop after two
    index.remove([removed.hex()])
    del stored[removed]
    assert check() == [2, 2, 0, 0, 2, 0]
    index.add([removed.hex()], [999])  # back, in a removed slot of the table
    stored[removed] = 999
    assert check() == [7, 5, 0, 0, 4, 0]
    assert len(index) == len(stored)
    assert _native.device_status() == 0


def test_index_refuses_more_keys_than_its_capacity():
    index = DevicePrefixIndex(capacity=4, block_size=4, device=DEV)
    keys = [k.hex() for k in block_keys(list(range(20)), 4)]
    index.add(keys[:4], [0, 1, 2, 3])
    with pytest.raises(RuntimeError, match="at most 4"):
        index.add(keys[4:], [4])
    with pytest.raises(ValueError, match="new and distinct"):
        index.add(keys[:1], [9])
