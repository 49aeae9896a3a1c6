"""Greedy decoding head: lm_head GEMM with the argmax in its epilogue (hb_lm_head_argmax).

The reference samples temperature-0 rows with ``torch.argmax`` over the bf16 logits
(src/helios/runtime/qwen3/decode.py:458-460, engine.py:472-473): the first largest id.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helios_b200 import _native, ops
from helios_b200.decode import Decoder
from helios_b200.paged_cache import KVPagePool, PagedKVCache

from tests.test_gpu_model import _model, _split

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.mark.parametrize("m,vocab,k", [(1, 151936, 2560), (33, 151936, 2560), (130, 4096, 256), (7, 1000, 128),
                                       (128, 384, 64)])
def test_integer_logits_match_torch_argmax_exactly(m, vocab, k):
    """Entries in {-1, 0, 1}: every logit is an exact integer in any summation order, so the bf16
    logits are the same as cuBLAS's and the ids must equal torch.argmax's, ties (frequent here)
    going to the lowest id."""
    g = torch.Generator(device=DEV).manual_seed(m + vocab)
    x = torch.randint(-1, 2, (m, k), device=DEV, generator=g).to(torch.bfloat16)
    w = torch.randint(-1, 2, (vocab, k), device=DEV, generator=g).to(torch.bfloat16)
    ids = ops.lm_head_argmax(x, w)
    want = F.linear(x, w).argmax(-1)
    assert ids.tolist() == want.tolist()
    again = ops.lm_head_argmax(x, w)  # the keys were left at zero: the next call starts clean
    assert again.tolist() == want.tolist()
    assert _native.device_status() == 0


def test_random_logits_pick_the_largest_bf16_logit():
    """Gaussian data at the Qwen3-4B head shape: fp32 sums in another order may round a logit to
    the neighbouring bf16 value, so the chosen id's cuBLAS logit must be within one bf16 step of
    the row maximum, and nearly every row must agree exactly."""
    g = torch.Generator(device=DEV).manual_seed(7)
    m, vocab, k = 64, 151936, 2560
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(vocab, k, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    ids = ops.lm_head_argmax(x, w)
    logits = F.linear(x, w).float()
    top = logits.max(-1).values
    step = torch.exp2(torch.floor(torch.log2(top.abs())) - 7)  # one bf16 step at the maximum
    chosen = logits.gather(1, ids[:, None]).squeeze(1)
    assert (chosen >= top - step).all()
    assert (ids == logits.argmax(-1)).float().mean() >= 0.95


@pytest.mark.parametrize("graphs", [False, True])
def test_greedy_continuation_matches_reference(golden_dir, graphs):
    """The golden mixed tick and its 64-step greedy continuation, sampled by the fused head."""
    g = np.load(golden_dir / "bf16_tick.npz")
    model = _model()
    if graphs:
        model.enable_cuda_graphs()
    decoder = Decoder(model)
    pool = decoder.page_pool = KVPagePool(model.config, 24, device=DEV)
    prompts = _split(g["prompts"].tolist(), g["prompt_lengths"].tolist())
    chunks = _split(g["chunks"].tolist(), g["chunk_lengths"].tolist())
    logit_counts = g["logit_counts"].tolist()
    steps = g["greedy"].shape[1]
    caches = []
    for prompt in prompts:
        cache = PagedKVCache(pool, len(prompt) + 320 + steps)
        decoder.packed_caches([cache], [prompt])
        caches.append(cache)
    caches.append(PagedKVCache(pool, 300 + steps))
    ids = decoder.packed_caches_greedy(caches, chunks, logit_counts=logit_counts)
    last = np.cumsum(logit_counts) - 1
    greedy = [ids[torch.as_tensor(last, device=DEV)].tolist()]
    for _ in range(steps - 1):
        greedy.append(decoder.packed_caches_greedy(caches, [[t] for t in greedy[-1]]).tolist())
    assert (np.array(greedy).T == g["greedy"]).all()
    assert _native.device_status() == 0


def test_decode_caches_greedy_is_the_argmax_of_decode_caches(golden_dir):
    g = np.load(golden_dir / "bf16_tick.npz")
    model = _model()
    decoder = Decoder(model)
    pool = decoder.page_pool = KVPagePool(model.config, 24, device=DEV)
    prompts = _split(g["prompts"].tolist(), g["prompt_lengths"].tolist())[:3]
    caches_a = [PagedKVCache(pool, len(p) + 8) for p in prompts]
    caches_b = [PagedKVCache(pool, len(p) + 8) for p in prompts]
    for ca, cb, p in zip(caches_a, caches_b, prompts):
        decoder.packed_caches([ca], [p])
        decoder.packed_caches([cb], [p])
    tokens = [5, 17, 4000]
    logits = decoder.decode_caches(caches_a, tokens)
    ids = decoder.decode_caches_greedy(caches_b, tokens)
    assert ids.tolist() == logits.argmax(-1).tolist()
    assert [c.length for c in caches_a] == [c.length for c in caches_b]


def test_nan_logits_win_at_their_lowest_id():
    """A NaN logit counts as the largest, as torch.argmax treats it; of several, the lowest id."""
    g = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randint(-1, 2, (5, 128), device=DEV, generator=g).to(torch.bfloat16)
    w = torch.randint(-1, 2, (1000, 128), device=DEV, generator=g).to(torch.bfloat16)
    w[700, 3] = float("nan")
    w[300, 5] = float("nan")
    ids = ops.lm_head_argmax(x, w)
    assert ids.tolist() == F.linear(x, w).argmax(-1).tolist() == [300] * 5
