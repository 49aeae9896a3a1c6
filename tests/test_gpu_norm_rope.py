"""Kernel (b) parity: fused q/k RMSNorm + RoPE + KV append vs the oracle.

The oracle follows the reference's rounding points (fp32 norm, bf16 round,
fp32 RoPE from the rounded value, bf16 round). The CUDA kernel may differ only
where the fp32 sum of squares or rsqrt rounds differently: at most one bf16 ulp,
on a small fraction of elements. V rows and plain appends must be bit-exact.
"""

import pytest
import torch

from helios_b200 import _native, ops
from oracle.numerics import apply_rope, rms_norm, rope_tables

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return (a.contiguous().view(torch.int16).int() - b.contiguous().view(torch.int16).int()).abs()


def _run_kernel(dim, rope: bool):
    heads, kv_heads, tokens, pages = 8, 2, 300, 8
    g = torch.Generator().manual_seed(0)
    qkv = torch.randn(tokens, (heads + 2 * kv_heads) * dim, generator=g).to(torch.bfloat16)
    positions = torch.randint(0, 4096, (tokens,), generator=g)
    slots = torch.randperm(pages * 256, generator=g)[:tokens]
    q_scale = (0.5 + torch.rand(dim, generator=g)).float()
    k_scale = (0.5 + torch.rand(dim, generator=g)).float()
    cos, sin = rope_tables(dim, 4096, 1e6)
    key_pool = torch.zeros(pages, 256, kv_heads, dim, dtype=torch.bfloat16, device=DEV)
    value_pool = torch.zeros_like(key_pool)
    d_qkv = qkv.to(DEV)
    q = d_qkv[:, : heads * dim].view(tokens, heads, dim)
    k = d_qkv[:, heads * dim: (heads + kv_heads) * dim].view(tokens, kv_heads, dim)
    v = d_qkv[:, (heads + kv_heads) * dim:].view(tokens, kv_heads, dim)
    q_out = torch.empty(tokens, heads, dim, dtype=torch.bfloat16, device=DEV)
    ops.qk_norm_rope_append(q, k, v, q_scale=q_scale.to(DEV), k_scale=k_scale.to(DEV), eps=1e-6,
                            cos=cos.to(DEV) if rope else None, sin=sin.to(DEV) if rope else None,
                            positions=positions.to(DEV), write_slots=slots.to(DEV), q_out=q_out,
                            key_pool=key_pool, value_pool=value_pool)
    assert _native.device_status() == 0
    qh = qkv[:, : heads * dim].view(tokens, heads, dim).transpose(0, 1)
    kh = qkv[:, heads * dim: (heads + kv_heads) * dim].view(tokens, kv_heads, dim).transpose(0, 1)
    vh = qkv[:, (heads + kv_heads) * dim:].view(tokens, kv_heads, dim)
    q_ref = rms_norm(qh, q_scale, 1e-6)
    k_ref = rms_norm(kh, k_scale, 1e-6)
    if rope:
        q_ref = apply_rope(q_ref, cos, sin, positions)
        k_ref = apply_rope(k_ref, cos, sin, positions)
    flat_k = key_pool.view(-1, kv_heads, dim).cpu()
    flat_v = value_pool.view(-1, kv_heads, dim).cpu()
    assert torch.equal(flat_v[slots], vh)
    untouched = torch.ones(pages * 256, dtype=torch.bool)
    untouched[slots] = False
    assert not flat_k[untouched].any() and not flat_v[untouched].any()
    return (q_out.cpu(), q_ref.transpose(0, 1)), (flat_k[slots], k_ref.transpose(0, 1))


@pytest.mark.parametrize("dim", [128, 64])
def test_norm_matches_oracle_within_one_ulp(dim):
    """The per-head RMSNorm alone: at most one bf16 ulp (fp32 reduction order, rsqrtf)."""
    for got, want in _run_kernel(dim, rope=False):
        ulps = _ulps(got, want)
        assert ulps.max().item() <= 1 and (ulps == 0).float().mean().item() > 0.98


@pytest.mark.parametrize("dim", [128, 64])
def test_norm_rope_append_matches_oracle(dim):
    """Norm + RoPE: x*cos + rot(x)*sin near cancellation can turn a one-ulp difference of the
    normalised input into several ulps of a small result, so the bound is two bf16 ulps of
    max(|result|, 1) -- the scale of the terms being added -- and almost every element exact."""
    for got, want in _run_kernel(dim, rope=True):
        diff = (got.float() - want.float()).abs()
        bound = 2 ** -6 * want.float().abs().clamp(min=1.0)
        assert (diff <= bound).all(), diff.max().item()
        assert (diff == 0).float().mean().item() > 0.97


def test_plain_append_is_exact_and_bad_slots_are_flagged():
    tokens, kv_heads, dim, pages = 64, 2, 128, 2
    k = torch.randn(tokens, kv_heads, dim, device=DEV).to(torch.bfloat16)
    v = torch.randn(tokens, kv_heads, dim, device=DEV).to(torch.bfloat16)
    key_pool = torch.zeros(pages, 256, kv_heads, dim, dtype=torch.bfloat16, device=DEV)
    value_pool = torch.zeros_like(key_pool)
    slots = torch.arange(tokens, device=DEV) * 3
    slots[5] = pages * 256 + 7  # outside the pool: skipped and reported, never written
    _native.device_status(clear=True)
    ops.qk_norm_rope_append(None, k, v, q_scale=None, k_scale=None, eps=0.0, cos=None, sin=None, positions=None,
                            write_slots=slots, q_out=None, key_pool=key_pool, value_pool=value_pool)
    status = _native.device_status(clear=True)
    assert "KV write slot outside the pool" in _native.describe_status(status)
    good = torch.ones(tokens, dtype=torch.bool, device=DEV)
    good[5] = False
    assert torch.equal(key_pool.view(-1, kv_heads, dim)[slots[good]], k[good])
    assert torch.equal(value_pool.view(-1, kv_heads, dim)[slots[good]], v[good])
