"""Device-resident prefix-cache index (the admission side of the reference's prefix cache).

The reference keys every 256-token block of a prompt by a SHA-256 chain over the block's
tokens as compact JSON (``hash_token_blocks``, src/helios/runtime/prefix_cache.py:86-110) and
``PrefixCache.longest_prefix`` (:208-222) walks those keys through a dict until the first
miss; both run in Python for every admitted request (about 0.8 ms per 4.7k-token prompt on
one host core). Here the keys of a whole batch of prompts are computed on the GPU
(``hb_hash_token_blocks``, one warp per prompt) and looked up in a device hash table
(``hb_prefix_index_lookup``) in the same stream, with one upload and one download.

* :func:`hash_token_blocks` returns the reference's hex keys for each prompt.
* :class:`DevicePrefixIndex` mirrors the set of stored block keys (with an int32 value each,
  e.g. the caller's handle of the cached block) on the device; ``lookup`` gives, per prompt,
  the keys and values of its leading full blocks that are stored, stopping at the first that
  is not, as ``longest_prefix`` does. The caller's ``PrefixCache`` keeps its own bookkeeping
  (hit counts, expiry, LRU order, memory) and tells the index what it stores and evicts.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from helios_b200 import _native

_MAX_TOKEN = 2 ** 31 - 1
_TORCH_DTYPES = {"u1": torch.uint8, "i4": torch.int32, "i8": torch.int64}


def _lib():
    return _native.load()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _flatten(token_lists: Sequence[Sequence[int]], block_size: int):
    """Host layout of a batch of prompts: int32 tokens, int64 token and block offsets, the
    number of full blocks per prompt. Same argument checks as the reference. Prompts may be
    lists of ints or integer arrays (numpy or CPU tensors, as a tokenizer returns them);
    arrays skip the per-token conversion of Python ints (~40 ns each)."""
    if block_size < 1:
        raise ValueError("block_size must be at least 1.")
    lengths = [len(t) for t in token_lists]
    offsets = np.zeros(len(lengths) + 1, dtype=np.int64)
    np.cumsum(lengths, out=offsets[1:])
    blocks = np.array([(n + block_size - 1) // block_size for n in lengths], dtype=np.int64)
    block_offsets = np.zeros(len(lengths) + 1, dtype=np.int64)
    np.cumsum(blocks, out=block_offsets[1:])
    full = np.array([n // block_size for n in lengths], dtype=np.int32)
    flat = np.empty(int(offsets[-1]), dtype=np.int32)
    for tokens, lo, n in zip(token_lists, offsets[:-1].tolist(), lengths):
        if not n:
            continue
        if isinstance(tokens, (np.ndarray, torch.Tensor)):
            part = np.asarray(tokens).reshape(-1)
            if part.dtype.kind not in "iu":
                raise ValueError("Token IDs must be non-negative integers.")
        else:
            part = np.fromiter(tokens, dtype=np.int64, count=n)
        if np.iinfo(part.dtype).max > _MAX_TOKEN and part.max() > _MAX_TOKEN:
            raise ValueError("Token IDs must be non-negative integers." if part.min() < 0
                             else "Token IDs above 2^31 - 1 are not supported.")
        flat[lo:lo + n] = part  # every value now fits int32 unchanged
    if flat.size and flat.min() < 0:
        raise ValueError("Token IDs must be non-negative integers.")
    return flat, offsets, block_offsets, full


class _PinnedStaging:
    """One grow-only pinned host buffer per device for the index's uploads: pinning fresh
    host memory on every call costs milliseconds, a reused buffer nothing. An event guards
    the buffer until the previous copy out of it has run."""

    def __init__(self) -> None:
        self.host: torch.Tensor | None = None
        self.event: torch.cuda.Event | None = None

    def take(self, nbytes: int) -> torch.Tensor:
        if self.event is not None:
            self.event.synchronize()
        if self.host is None or self.host.numel() < nbytes:
            self.host = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, pin_memory=True)
        return self.host[:nbytes]

    def done(self, device: torch.device) -> None:
        if self.event is None:
            self.event = torch.cuda.Event()
        self.event.record(torch.cuda.current_stream(device))


_STAGING: dict[torch.device, _PinnedStaging] = {}


def _upload(arrays: Sequence[np.ndarray], device: torch.device) -> list[torch.Tensor]:
    """One pinned host buffer and one copy for all of ``arrays`` (each 8-byte aligned)."""
    sizes = [(a.nbytes + 7) // 8 * 8 for a in arrays]
    staging = _STAGING.setdefault(device, _PinnedStaging())
    host = staging.take(max(8, sum(sizes)))
    at = 0
    for a, n in zip(arrays, sizes):
        host[at:at + a.nbytes].numpy()[:] = a.view(np.uint8).reshape(-1)
        at += n
    dev = host.to(device, non_blocking=True)
    staging.done(device)
    out, at = [], 0
    for a, n in zip(arrays, sizes):
        out.append(dev[at:at + a.nbytes].view(_TORCH_DTYPES[a.dtype.str[1:]]))
        at += n
    return out


def _hash(token_lists, block_size, device, words_per_block: int = 0, words: int = 0):
    """Digests of every block. They lead a device buffer (returned last) with room after them
    for ``words_per_block`` int32 per block plus ``words`` more, which the caller fills, so a
    single download brings everything back."""
    tokens, offsets, block_offsets, full = _flatten(token_lists, block_size)
    d_tokens, d_offsets, d_boffs, d_full = _upload([tokens, offsets, block_offsets, full], device)
    blocks = int(block_offsets[-1])
    buffer = torch.empty(blocks * 32 + 4 * (words_per_block * blocks + words), dtype=torch.uint8, device=device)
    digests = buffer[:blocks * 32].view(blocks, 32)
    if blocks:  # no tokens at all: nothing to key (and empty buffers have no address)
        rc = _lib().hb_hash_token_blocks(d_tokens.data_ptr(), d_offsets.data_ptr(), len(token_lists), block_size,
                                         d_boffs.data_ptr(), digests.data_ptr(), _stream(device))
        _native.check(rc, "hb_hash_token_blocks")
    return digests, d_boffs, d_full, block_offsets, full, buffer


def _hex_rows(digests: np.ndarray, lo: int, hi: int) -> list[str]:
    """Hex keys of digest rows lo..hi of a [blocks, 32] uint8 array."""
    text = digests[lo:hi].tobytes().hex()
    return [text[64 * i:64 * (i + 1)] for i in range(hi - lo)]


def hash_token_blocks(token_lists: Sequence[Sequence[int]], block_size: int,
                      device: torch.device | None = None) -> list[list[str]]:
    """Hex keys of every block of every prompt (partial last blocks included), equal to
    ``[b.hash for b in build_token_blocks(tokens, block_size)]`` of the reference."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    digests, _, _, block_offsets, _, _ = _hash(token_lists, block_size, device)
    host = digests.cpu().numpy()
    return [_hex_rows(host, int(block_offsets[p]), int(block_offsets[p + 1])) for p in range(len(token_lists))]


class DevicePrefixIndex:
    """The stored block keys of a prefix cache, on the device, with an int32 value per key."""

    def __init__(self, capacity: int, block_size: int, device: torch.device | None = None) -> None:
        if capacity < 1:
            raise ValueError("capacity must be at least 1.")
        if block_size < 1:
            raise ValueError("block_size must be at least 1.")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.block_size = block_size
        self.capacity = capacity
        slots = 1
        while slots < 2 * capacity:  # load factor at most 1/2
            slots *= 2
        self.slots = slots
        self.table = torch.zeros((slots, 12), dtype=torch.int32, device=self.device)
        self._values: dict[str, int] = {}

    def __len__(self) -> int:
        return len(self._values)

    def __contains__(self, key: str) -> bool:
        return key in self._values

    def add(self, keys: Sequence[str], values: Sequence[int]) -> None:
        """Store ``keys`` (hex block keys, not yet stored) with their ``values``."""
        if len(keys) != len(values):
            raise ValueError("Each key needs one value.")
        if len(set(keys)) != len(keys) or any(k in self._values for k in keys):
            raise ValueError("Keys must be new and distinct.")
        if len(self._values) + len(keys) > self.capacity:
            raise RuntimeError(f"Prefix index holds at most {self.capacity} keys.")
        if not keys:
            return
        raw = np.frombuffer(b"".join(bytes.fromhex(k) for k in keys), dtype=np.uint8)
        vals = np.asarray(values, dtype=np.int32)
        d_raw, d_vals = _upload([raw, vals], self.device)
        rc = _lib().hb_prefix_index_insert(self.table.data_ptr(), self.slots, d_raw.data_ptr(), d_vals.data_ptr(),
                                           len(keys), _stream(self.device))
        _native.check(rc, "hb_prefix_index_insert")
        self._values.update(zip(keys, (int(v) for v in values)))

    def remove(self, keys: Sequence[str]) -> None:
        """Drop ``keys`` (evicted or expired blocks); keys not stored are ignored."""
        keys = [k for k in dict.fromkeys(keys) if k in self._values]
        if not keys:
            return
        raw = np.frombuffer(b"".join(bytes.fromhex(k) for k in keys), dtype=np.uint8)
        (d_raw,) = _upload([raw], self.device)
        rc = _lib().hb_prefix_index_remove(self.table.data_ptr(), self.slots, d_raw.data_ptr(), len(keys),
                                           _stream(self.device))
        _native.check(rc, "hb_prefix_index_remove")
        for k in keys:
            del self._values[k]

    def lookup(self, token_lists: Sequence[Sequence[int]]) -> list[tuple[list[str], list[int]]]:
        """Per prompt, the keys and values of its leading full blocks that are stored, up to the
        first that is not (``PrefixCache.longest_prefix``'s walk)."""
        prompts = len(token_lists)
        # Digests, values and match counts side by side, so one download brings all three back.
        digests, d_boffs, d_full, block_offsets, full, out = _hash(token_lists, self.block_size, self.device,
                                                                   words_per_block=1, words=prompts)
        blocks = int(block_offsets[-1])
        if blocks == 0:
            return [([], []) for _ in range(prompts)]
        values = out[blocks * 32:blocks * 36].view(torch.int32)
        matched = out[blocks * 36:].view(torch.int32)  # every entry written by the kernel
        rc = _lib().hb_prefix_index_lookup(self.table.data_ptr(), self.slots, digests.data_ptr(), d_boffs.data_ptr(),
                                           d_full.data_ptr(), prompts, matched.data_ptr(), values.data_ptr(),
                                           _stream(self.device))
        _native.check(rc, "hb_prefix_index_lookup")
        raw = out.cpu().numpy()
        host = raw[:blocks * 32].reshape(blocks, 32)
        vals = raw[blocks * 32:blocks * 36].view(np.int32)
        counts = raw[blocks * 36:].view(np.int32).tolist()
        starts = block_offsets[:-1].tolist()
        return [(_hex_rows(host, lo, lo + n), vals[lo:lo + n].tolist()) for lo, n in zip(starts, counts)]
