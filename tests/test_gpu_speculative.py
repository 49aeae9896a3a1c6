"""Speculative verification on the device (hb_verify_drafts, decode.sample_and_verify)
against the oracle restatement of Engine._execute_batch's acceptance loop
(src/helios/runtime/engine.py:488-520): accepted counts and emitted tokens must be
identical, and drafted rows' caches truncated to length + 1 + accepted."""

import pytest
import torch

from helios_b200 import _native, ops
from helios_b200.config import Qwen3Config, Sampling
from helios_b200.decode import Decoder, sample_and_verify
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool, PagedKVCache
from oracle.speculative import accept

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
GREEDY = Sampling(max_new_tokens=64, temperature=0.0, top_p=1.0)


def test_kernel_matches_oracle_on_random_drafts():
    g = torch.Generator().manual_seed(0)
    rows, vocab = 300, 512
    counts = torch.randint(1, 17, (rows,), generator=g).tolist()
    logit_counts = [c if torch.rand(1, generator=g).item() < 0.7 else 1 for c in counts]
    logits = torch.randn(sum(logit_counts), vocab, generator=g).to(torch.bfloat16)
    predictions = logits.float().argmax(-1).tolist()
    chunks, at = [], 0
    for c, lc in zip(counts, logit_counts):
        chunk = torch.randint(0, vocab, (c,), generator=g).tolist()
        if lc > 1:  # drafts that follow the predictions for a random number of steps
            keep = torch.randint(0, lc, (1,), generator=g).item()
            for i in range(keep):
                chunk[c - lc + 1 + i] = predictions[at + i]
        chunks.append(chunk)
        at += lc
    # The trailing logit rows of a row hold its last lc tokens; the oracle's chunk is those.
    want_acc, want_emit = accept([ch[len(ch) - lc:] for ch, lc in zip(chunks, logit_counts)], logit_counts,
                                 predictions)
    tokens = torch.tensor([t for ch in chunks for t in ch], device=DEV)
    cu = torch.tensor([0] + torch.tensor(counts).cumsum(0).tolist(), dtype=torch.int32, device=DEV)
    offsets = torch.tensor([0] + torch.tensor(logit_counts).cumsum(0).tolist(), dtype=torch.int32, device=DEV)
    accepted, emitted = ops.verify_drafts(tokens, cu, offsets, torch.tensor(predictions, device=DEV))
    assert accepted.tolist() == want_acc
    flat, starts = emitted.tolist(), offsets.tolist()
    assert [flat[starts[r]: starts[r] + want_acc[r] + 1] for r in range(rows)] == want_emit
    assert sum(a > 0 for a in want_acc) > 20 and _native.device_status() == 0


def test_drafted_tick_through_the_model():
    """A draft equal to the model's own greedy continuation is accepted in full (plus the
    bonus token); an arbitrary draft stops where it first differs; drafted rows' caches are
    truncated to length + 1 + accepted."""
    torch.manual_seed(0)
    shape = dict(vocab_size=4096, context_length=4096, hidden_size=512, n_heads=8, n_layers=2, hidden_dim=1024,
                 head_dim=128, n_kv_heads=2, rope_base=1e6, rms_norm_eps=1e-6, dtype=torch.bfloat16)
    model = Qwen3Model(Qwen3Config(**shape)).to(DEV).eval()
    decoder = Decoder(model)
    pool = decoder.page_pool = KVPagePool(model.config, 24, device=DEV)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (60, 130)]
    caches = [PagedKVCache(pool, 400) for _ in prompts]
    heads = sample_and_verify(decoder.packed_caches(caches, prompts), prompts, [1, 1], [GREEDY, GREEDY])
    lengths = [c.length for c in caches]
    row0 = [heads[0][0], 0, 0, 0]
    row1 = [heads[1][0], 1, 2, 3]  # arbitrary drafts
    # Logit row k of a drafted row depends only on its tokens up to k (causal), so each
    # pass fixes one more draft of row 0 to the model's greedy id; the caches roll back.
    for k in range(3):
        logits = decoder.packed_caches(caches, [row0, row1], logit_counts=[4, 4])
        row0[k + 1] = int(logits[k].float().argmax().item())
        for cache, length in zip(caches, lengths):
            cache.truncate(length)
    logits = decoder.packed_caches(caches, [row0, row1], logit_counts=[4, 4])
    predictions = logits.float().argmax(-1).tolist()
    emitted = sample_and_verify(logits, [row0, row1], [4, 4], [GREEDY, GREEDY], caches=caches,
                                cache_lengths=lengths)
    acc, want = accept([row0, row1], [4, 4], predictions)
    assert acc[0] == 3 and emitted[0] == row0[1:] + [predictions[3]]  # 3 drafts + the bonus token
    assert emitted == want
    assert [c.length for c in caches] == [lengths[0] + 1 + acc[0], lengths[1] + 1 + acc[1]]
    assert _native.device_status() == 0
