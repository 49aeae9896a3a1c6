"""End-to-end parity of the packed tick: B200 model vs the reference's outputs.

``tests/golden/bf16_tick.npz`` holds the reference's packed-path logits for a
mixed tick (decode rows, a drafted row, a continued chunk and a fresh prefill)
at the Qwen3-4B head shape, and its greedy continuation for 64 steps. The B200
model loads the reference's seed-0 random-init weights (rebuilt by the oracle,
whose weight construction the CPU suite pins against the reference), replays
the same prompts through paged prefill ticks, and must give logits within 2 bf16
ulps of each row's largest logit and identical greedy ids.
"""

import numpy as np
import pytest
import torch

from helios_b200 import _native
from helios_b200.config import Qwen3Config, Sampling
from helios_b200.decode import Decoder, sample_rows
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool, PagedKVCache
from oracle.model import OracleConfig, build_state_dict

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
SHAPE = dict(vocab_size=4096, context_length=4096, hidden_size=512, n_heads=8, n_layers=2, hidden_dim=1024,
             head_dim=128, n_kv_heads=2, rope_base=1e6, rms_norm_eps=1e-6, dtype=torch.bfloat16)


def _ulp(x: torch.Tensor) -> torch.Tensor:
    """bf16 spacing (8 significand bits) at magnitude ``x``."""
    return torch.exp2(torch.floor(torch.log2(x.clamp(min=torch.finfo(torch.float32).tiny))) - 7)


def _split(flat, lengths):
    out, at = [], 0
    for n in lengths:
        out.append(flat[at:at + n])
        at += n
    return out


def _model():
    model = Qwen3Model(Qwen3Config(**SHAPE))
    model.load_state_dict(build_state_dict(OracleConfig(**SHAPE), 0), strict=False)
    return model.to(DEV).eval()


def test_weights_match_reference_init():
    """The module tree is created in the reference's order: seed 0 gives its weights."""
    torch.manual_seed(0)
    model = Qwen3Model(Qwen3Config(**SHAPE))
    mine = model.state_dict()
    for key, value in build_state_dict(OracleConfig(**SHAPE), 0).items():
        assert torch.equal(mine[key], value), key


def test_mixed_tick_logits_and_greedy_match_reference(golden_dir):
    g = np.load(golden_dir / "bf16_tick.npz")
    model = _model()
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
    logits = decoder.packed_caches(caches, chunks, logit_counts=logit_counts).float().cpu()
    ref = torch.from_numpy(g["logits"])
    diff = (logits - ref).abs().max(-1).values
    ulp = _ulp(ref.abs().max(-1).values)
    print(f"bf16 tick logits vs reference: max {float((diff / ulp).max()):.3f} ulp of the row max")
    assert (diff <= 2 * ulp).all(), diff / ulp
    last = np.cumsum(logit_counts) - 1
    heads = logits[torch.as_tensor(last)]
    greedy, maxima = [heads.argmax(-1).tolist()], [heads.max(-1).values.tolist()]
    for _ in range(steps - 1):
        out = decoder.packed_caches(caches, [[t] for t in greedy[-1]]).float()
        greedy.append(out.argmax(-1).tolist())
        maxima.append(out.max(-1).values.tolist())
    assert (np.array(greedy).T == g["greedy"]).all()
    # The winning logit of every row at every step tracks the reference's, within 2 ulps.
    want = torch.from_numpy(g["greedy_max"])
    err = (torch.tensor(maxima).T - want).abs() / _ulp(want.abs())
    print(f"winning logits over {steps} steps: max {float(err.max()):.3f} ulp")
    assert (err <= 2).all()
    assert [p.index for c in caches for p in c.pages] == g["page_tables"].tolist()
    assert _native.device_status() == 0


def test_decode_caches_and_fused_greedy_sampler_agree_with_packed_path(golden_dir):
    """A decode-only tick (PagedBatchCache.prepare(1)) gives the packed path's logits."""
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
    packed = decoder.packed_caches(caches_a, [[t] for t in tokens]).float()
    decoded = decoder.decode_caches(caches_b, tokens).float()
    torch.testing.assert_close(decoded, packed, rtol=0, atol=0)
    ids = sample_rows(decoded.to(torch.bfloat16), [Sampling(temperature=0, top_p=1, max_new_tokens=1)] * 3)
    assert ids.tolist() == decoded.argmax(-1).tolist()
