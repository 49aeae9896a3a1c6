"""Fused q|k|v projection + kernel (b) (hb_gemm_qkv_norm_rope_append) against the reference.

The expected values take torch's GEMM for the projection (bf16 outputs, as the reference's
three nn.Linear return) and the oracle's RMSNorm and RoPE (the reference's rounding points).
The fused kernel accumulates K in a different order, so a projection output can land one bf16
ulp away; the norm and the rotation then carry that difference. Bounds: value rows within one
bf16 ulp, q/k rows within the norm/RoPE kernel's bound (two bf16 ulps of max(|result|, 1)),
and most elements exact. Shapes: one token, ragged M tiles, the config-3 tick shape.
"""

import pytest
import torch
import torch.nn.functional as F

from helios_b200 import _native, ops
from oracle.numerics import apply_rope, rms_norm, rope_tables

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
D = 128


def _inputs(m, heads, kv_heads, hidden, pages, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, hidden, generator=g).to(torch.bfloat16)
    w = (torch.randn((heads + 2 * kv_heads) * D, hidden, generator=g) / hidden ** 0.5).to(torch.bfloat16)
    positions = torch.randint(0, 4096, (m,), generator=g)
    slots = torch.randperm(pages * 256, generator=g)[:m]
    q_scale = (0.5 + torch.rand(D, generator=g)).float()
    k_scale = (0.5 + torch.rand(D, generator=g)).float()
    return x, w, positions, slots, q_scale, k_scale


def _fused(x, w, positions, slots, q_scale, k_scale, cos, sin, heads, kv_heads, pages, half_tables=False):
    key_pool = torch.zeros(pages, 256, kv_heads, D, dtype=torch.bfloat16, device=DEV)
    value_pool = torch.zeros_like(key_pool)
    q_out = torch.empty(x.shape[0], heads, D, dtype=torch.bfloat16, device=DEV)
    ops.gemm_qkv_norm_rope_append(x.to(DEV), w.to(DEV), heads=heads, kv_heads=kv_heads, q_scale=q_scale.to(DEV),
                                  k_scale=k_scale.to(DEV), eps=1e-6, cos=cos.to(DEV), sin=sin.to(DEV),
                                  positions=positions.to(DEV), write_slots=slots.to(DEV), q_out=q_out,
                                  key_pool=key_pool, value_pool=value_pool, rope_half_tables=half_tables)
    return q_out.cpu(), key_pool.view(-1, kv_heads, D).cpu(), value_pool.view(-1, kv_heads, D).cpu()


def _close(got, want, bound_scale):
    diff = (got.float() - want.float()).abs()
    bound = bound_scale * want.float().abs().clamp(min=1.0)
    assert (diff <= bound).all(), diff.max().item()
    assert (diff == 0).float().mean().item() > 0.9


def _full_tables():
    """Rope tables whose halves differ, for the path that reads whole rows."""
    cos, sin = rope_tables(D, 4096, 1e6)
    return cos, torch.cat((sin[:, D // 2:], -sin[:, :D // 2]), dim=1)


@pytest.mark.parametrize("half_tables", [True, False])
@pytest.mark.parametrize("m,heads,kv_heads,hidden", [(1, 4, 2, 256), (300, 8, 2, 512), (2080, 32, 8, 2560)])
def test_fused_qkv_matches_projection_then_norm_rope(m, heads, kv_heads, hidden, half_tables):
    pages = (m + 255) // 256 + 2
    x, w, positions, slots, q_scale, k_scale = _inputs(m, heads, kv_heads, hidden, pages, m + hidden)
    cos, sin = rope_tables(D, 4096, 1e6) if half_tables else _full_tables()
    q_got, k_flat, v_flat = _fused(x, w, positions, slots, q_scale, k_scale, cos, sin, heads, kv_heads, pages,
                                   half_tables)
    assert _native.device_status() == 0

    qkv = F.linear(x.to(DEV), w.to(DEV)).cpu()  # bf16, as the three projections return
    qh = qkv[:, : heads * D].view(m, heads, D).transpose(0, 1)
    kh = qkv[:, heads * D: (heads + kv_heads) * D].view(m, kv_heads, D).transpose(0, 1)
    vh = qkv[:, (heads + kv_heads) * D:].view(m, kv_heads, D)
    q_want = apply_rope(rms_norm(qh, q_scale, 1e-6), cos, sin, positions).transpose(0, 1)
    k_want = apply_rope(rms_norm(kh, k_scale, 1e-6), cos, sin, positions).transpose(0, 1)

    _close(v_flat[slots], vh, 2 ** -7)  # one bf16 ulp of a projection output
    _close(q_got, q_want, 2 ** -6)
    _close(k_flat[slots], k_want, 2 ** -6)
    untouched = torch.ones(k_flat.shape[0], dtype=torch.bool)
    untouched[slots] = False
    assert not k_flat[untouched].any() and not v_flat[untouched].any()


@pytest.mark.parametrize("half_tables", [True, False])
def test_fused_qkv_equals_separate_kernels_on_the_same_projection(half_tables):
    """Fed projection values that every accumulation order gets exactly (one-hot rows of x),
    the fused epilogue writes the same bits as kernel (b): both run the same per-lane norm
    and RoPE arithmetic with the same fp32 summation order."""
    m, heads, kv_heads, hidden, pages = 200, 4, 2, 128, 2
    g = torch.Generator().manual_seed(7)
    # x one-hot per row: x @ w^T selects a weight column, so every projection output is exact.
    cols = torch.randint(0, hidden, (m,), generator=g)
    x = torch.zeros(m, hidden, dtype=torch.bfloat16)
    x[torch.arange(m), cols] = 1
    w = torch.randn((heads + 2 * kv_heads) * D, hidden, generator=g).to(torch.bfloat16)
    positions = torch.randint(0, 4096, (m,), generator=g)
    slots = torch.randperm(pages * 256, generator=g)[:m]
    q_scale = (0.5 + torch.rand(D, generator=g)).float()
    k_scale = (0.5 + torch.rand(D, generator=g)).float()
    cos, sin = rope_tables(D, 4096, 1e6) if half_tables else _full_tables()
    q_got, k_flat, v_flat = _fused(x, w, positions, slots, q_scale, k_scale, cos, sin, heads, kv_heads, pages,
                                   half_tables)

    qkv = w.t()[cols].contiguous().to(DEV)  # the exact projection
    q = qkv[:, : heads * D].view(m, heads, D)
    k = qkv[:, heads * D: (heads + kv_heads) * D].view(m, kv_heads, D)
    v = qkv[:, (heads + kv_heads) * D:].view(m, kv_heads, D)
    key_pool = torch.zeros(pages, 256, kv_heads, D, dtype=torch.bfloat16, device=DEV)
    value_pool = torch.zeros_like(key_pool)
    q_out = torch.empty(m, heads, D, dtype=torch.bfloat16, device=DEV)
    ops.qk_norm_rope_append(q, k, v, q_scale=q_scale.to(DEV), k_scale=k_scale.to(DEV), eps=1e-6, cos=cos.to(DEV),
                            sin=sin.to(DEV), positions=positions.to(DEV), write_slots=slots.to(DEV), q_out=q_out,
                            key_pool=key_pool, value_pool=value_pool)
    assert _native.device_status() == 0
    assert torch.equal(v_flat, value_pool.view(-1, kv_heads, D).cpu())
    assert torch.equal(k_flat, key_pool.view(-1, kv_heads, D).cpu())
    assert torch.equal(q_got, q_out.cpu())


def test_bad_write_slot_is_flagged_and_skipped():
    m, heads, kv_heads, hidden, pages = 130, 4, 2, 256, 2
    x, w, positions, slots, q_scale, k_scale = _inputs(m, heads, kv_heads, hidden, pages, 11)
    slots[129] = pages * 256  # one past the pool
    cos, sin = rope_tables(D, 4096, 1e6)
    _native.device_status(clear=True)
    _, k_flat, v_flat = _fused(x, w, positions, slots, q_scale, k_scale, cos, sin, heads, kv_heads, pages)
    status = _native.device_status(clear=True)
    assert "KV write slot outside the pool" in _native.describe_status(status)
    written = (k_flat.abs().sum((1, 2)) > 0).sum().item()
    assert written == m - 1


def test_rejects_unsupported_shapes():
    x = torch.zeros(4, 256, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(8 * 64, 256, device=DEV, dtype=torch.bfloat16)
    pool = torch.zeros(1, 256, 2, 64, device=DEV, dtype=torch.bfloat16)
    q_out = torch.empty(4, 4, 64, device=DEV, dtype=torch.bfloat16)
    slots = torch.zeros(4, dtype=torch.long, device=DEV)
    with pytest.raises(ValueError, match="hb_gemm_qkv_norm_rope_append"):
        ops.gemm_qkv_norm_rope_append(x, w, heads=4, kv_heads=2, q_scale=None, k_scale=None, eps=1e-6, cos=None,
                                      sin=None, positions=None, write_slots=slots, q_out=q_out, key_pool=pool,
                                      value_pool=pool)


@pytest.mark.parametrize("half_tables", [True, False])
def test_rope_gather_rows(half_tables):
    """[w / 4, T, 4] per-token rows of the tables; zeros for positions outside them."""
    cos, sin = rope_tables(D, 512, 1e6)
    positions = torch.tensor([0, 5, 511, 512, -1, 77], dtype=torch.long)
    got_c, got_s = ops.rope_gather(cos.to(DEV), sin.to(DEV), positions.to(DEV), half_tables=half_tables)
    width = D // 2 if half_tables else D
    ok = (positions >= 0) & (positions < 512)
    for got, table in ((got_c, cos), (got_s, sin)):
        want = torch.zeros(positions.numel(), width)
        want[ok] = table[positions[ok], :width]
        assert torch.equal(got.cpu().permute(1, 0, 2).reshape(positions.numel(), width), want)


def test_model_tick_with_fused_qkv_matches_unfused(monkeypatch):
    """The model with the fused q|k|v route switched on gives the unfused route's logits for a
    300-token prefill tick (within the model tests' bf16 bound: the projections' accumulation
    order differs)."""
    from helios_b200 import model as model_mod
    from helios_b200.config import Qwen3Config
    from helios_b200.decode import Decoder
    from helios_b200.paged_cache import KVPagePool, PagedKVCache

    shape = dict(vocab_size=4096, context_length=4096, hidden_size=512, n_heads=8, n_layers=2, hidden_dim=1024,
                 head_dim=128, n_kv_heads=2, rope_base=1e6, rms_norm_eps=1e-6, dtype=torch.bfloat16)
    torch.manual_seed(0)
    model = model_mod.Qwen3Model(Qwen3Config(**shape)).to(DEV).eval()
    assert model.rope_half_tables
    prompts = [torch.randint(0, 4096, (n,), generator=torch.Generator().manual_seed(n)).tolist() for n in (300, 40)]

    def run():
        decoder = Decoder(model)
        decoder.page_pool = KVPagePool(model.config, 8, device=DEV)
        caches = [PagedKVCache(decoder.page_pool, 512) for _ in prompts]
        return decoder.packed_caches(caches, prompts).float().cpu()

    monkeypatch.setattr(model_mod, "FUSED_QKV_MIN_ROWS", None)
    want = run()
    monkeypatch.setattr(model_mod, "FUSED_QKV_MIN_ROWS", 256)
    got = run()
    assert _native.device_status() == 0
    diff = (got - want).abs().max(-1).values
    assert (diff <= 2e-2 * want.abs().max(-1).values).all(), diff
