"""CUDA-graph replay of ticks (helios_b200.graphs) against eager ticks.

Two decoders over twin pools see the same requests and token ids; one runs every
tick eagerly, the other replays the device half of each tick from CUDA graphs, with
attention launches sized to capacities and the tick's work counts read from the
device. Covered: a prefill tick, decode ticks whose rows cross split boundaries (the
work list changes under one graph), a new request joining with a prefill chunk (new
shape: a new capture), and uniform decode ticks (PagedBatchCache). The logits must
agree within the parity tolerance of the model tests and the greedy ids exactly.
"""

import pytest
import torch

from helios_b200 import _native
from helios_b200.config import Qwen3Config
from helios_b200.decode import Decoder
from helios_b200.model import Qwen3Model
from helios_b200.paged_cache import KVPagePool, PagedKVCache

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
SHAPE = dict(vocab_size=4096, context_length=4096, hidden_size=512, n_heads=8, n_layers=2, hidden_dim=1024,
             head_dim=128, n_kv_heads=2, rope_base=1e6, rms_norm_eps=1e-6, dtype=torch.bfloat16)


def _close(graphed: torch.Tensor, eager: torch.Tensor) -> None:
    scale = eager.float().abs().amax(dim=-1, keepdim=True).clamp(min=1.0)
    assert ((graphed.float() - eager.float()).abs() <= 2e-2 * scale).all()
    assert torch.equal(graphed.argmax(-1), eager.argmax(-1))


def test_graph_ticks_match_eager_ticks():
    torch.manual_seed(0)
    model = Qwen3Model(Qwen3Config(**SHAPE)).to(DEV).eval()
    model.enable_cuda_graphs()
    runner = model._graphs
    eager, graphed = Decoder(model), Decoder(model)
    pools = [KVPagePool(model.config, 48, device=DEV) for _ in range(2)]
    eager.page_pool, graphed.page_pool = pools

    def tick(caches_e, caches_g, chunks):
        model._graphs = None
        a = eager.packed_caches(caches_e, chunks).clone()
        model._graphs = runner
        b = graphed.packed_caches(caches_g, chunks).clone()
        _close(b, a)
        return a.argmax(-1).tolist()

    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (200, 250, 40)]
    caps = [n + 700 for n in (200, 250, 40)]
    ce = [PagedKVCache(pools[0], c) for c in caps]
    cg = [PagedKVCache(pools[1], c) for c in caps]
    last = tick(ce, cg, prompts)
    for step in range(70):  # rows cross the 256-key split boundary at different steps
        chunks = [[t] for t in last]
        if step == 30:  # a new request joins with a prefill chunk: a new tick shape
            joined = torch.randint(0, 4096, (96,), generator=g).tolist()
            ce.append(PagedKVCache(pools[0], 900))
            cg.append(PagedKVCache(pools[1], 900))
            chunks.append(joined)
        last = tick(ce, cg, chunks)
    assert runner.captures >= 2 and runner.replays >= 60
    assert _native.device_status() == 0

    # Uniform decode ticks through decode_caches (PagedBatchCache).
    before = runner.replays
    for _ in range(6):
        model._graphs = None
        a = eager.decode_caches(ce, last).clone()
        model._graphs = runner
        b = graphed.decode_caches(cg, last).clone()
        _close(b, a)
        last = a.argmax(-1).tolist()
    assert runner.replays > before
    assert _native.device_status() == 0


def test_graph_ticks_with_a_shared_prefix_match_eager_ticks():
    """Decode rows that restored the same prefix pages (page aliasing) run their shared keys as
    prefix items on the tensor cores: replayed graphs read the prefix items' count from the
    device like the other work counts and must agree with eager ticks."""
    torch.manual_seed(0)
    model = Qwen3Model(Qwen3Config(**SHAPE)).to(DEV).eval()
    model.enable_cuda_graphs()
    runner = model._graphs
    eager, graphed = Decoder(model), Decoder(model)
    pools = [KVPagePool(model.config, 64, device=DEV) for _ in range(2)]
    eager.page_pool, graphed.page_pool = pools
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, 4096, (1100,), generator=g).tolist()
    bases = [PagedKVCache(pool, 1200) for pool in pools]
    model._graphs = None
    for dec, base in zip((eager, graphed), bases):
        dec.packed_caches([base], [prompt])
    blocks = [base.snapshot_block(0, 4 * 256) for base in bases]
    tails = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (5, 90, 260, 31, 140)]
    rows = [[], []]
    for side in range(2):
        for tail in tails:
            cache = PagedKVCache(pools[side], 1024 + len(tail) + 40)
            cache.restore_blocks([blocks[side]])
            rows[side].append(cache)
    a = eager.packed_caches(rows[0], tails).clone()
    b = graphed.packed_caches(rows[1], tails).clone()
    _close(b, a)
    last = a.argmax(-1).tolist()
    for _ in range(12):
        chunks = [[t] for t in last]
        model._graphs = None
        a = eager.packed_caches(rows[0], chunks).clone()
        model._graphs = runner
        b = graphed.packed_caches(rows[1], chunks).clone()
        assert graphed._packed_batch.num_prefix_items > 0  # the 5 rows share 4 pages
        _close(b, a)
        last = a.argmax(-1).tolist()
    assert runner.replays >= 10
    assert _native.device_status() == 0


def test_pipelined_decode_steps_match_synchronous_steps():
    """``workloads.decode_steps`` pipelined (the next tick takes the sampled ids on the device and
    is queued before the host reads them back) samples the same ids as the synchronous loop that
    reads every step's ids before queueing the next, over graph-replayed sampled decode ticks."""
    from helios_b200.config import Sampling
    from helios_b200.decode import sample_rows
    from helios_b200.workloads import decode_steps

    torch.manual_seed(0)
    model = Qwen3Model(Qwen3Config(**SHAPE)).to(DEV).eval()
    model.enable_cuda_graphs()
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (120, 300, 45, 260)]
    samplings = [Sampling(temperature=0.7, top_p=0.9, max_new_tokens=64)] * len(prompts)
    results = []
    for pipelined in (False, True):
        decoder = Decoder(model)
        decoder.page_pool = KVPagePool(model.config, 48, device=DEV)
        caches = [PagedKVCache(decoder.page_pool, len(p) + 40) for p in prompts]
        heads = decoder.packed_caches(caches, prompts).clone()
        gen = torch.Generator(device=DEV).manual_seed(5)
        first = sample_rows(heads, samplings, generator=gen).tolist()

        def tick(ids, caches=caches, gen=gen, decoder=decoder):
            return sample_rows(decoder.decode_caches(caches, ids), samplings, generator=gen)

        results.append([first] + decode_steps(tick, first, 24, pipelined))
        assert [c.length for c in caches] == [len(p) + 24 for p in prompts]
    assert results[0] == results[1]
    assert _native.device_status() == 0
