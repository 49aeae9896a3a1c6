"""Fused gate|up projection + SwiGLU (hb_gemm_swiglu) against the reference's formula.

The reference (FeedForward.forward, layers.py:26-27) rounds each projection output to
bf16, computes silu in fp32 from it, rounds, then multiplies and rounds. The expected
values use torch's own GEMM for the projections; the fused kernel accumulates K in a
different order, so a projection can land one bf16 ulp away and move the result by a
few ulps: the bound is the model tests' bf16 tolerance, and most elements must match
exactly. Shapes: partial M tiles, several column tiles and the config-3 tick shape.
"""

import pytest
import torch
import torch.nn.functional as F

from helios_b200 import _native, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _reference(x, w):
    inter = w.shape[0] // 2
    gate_up = F.linear(x, w)  # bf16 outputs, as each nn.Linear returns
    gate, up = gate_up[:, :inter], gate_up[:, inter:]
    return F.silu(gate.float()).to(torch.bfloat16) * up


@pytest.mark.parametrize("m,k,inter", [(1, 256, 128), (257, 512, 384), (2080, 2560, 9728)])
def test_fused_gate_up_swiglu_matches_reference(m, k, inter):
    g = torch.Generator(device=DEV).manual_seed(m + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * inter, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    got = ops.gemm_swiglu(x, w)
    want = _reference(x, w)
    torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)
    assert (got == want).float().mean().item() > 0.9
    assert _native.device_status() == 0


def test_rejects_unsupported_shapes():
    x = torch.zeros(4, 100, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(256, 100, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="hb_gemm_swiglu"):
        ops.gemm_swiglu(x, w)


@pytest.mark.parametrize("rows", [100, 1300])
def test_feed_forward_takes_either_path_with_the_same_result(rows, monkeypatch):
    """FeedForward switches to the fused kernel from FUSED_GATE_UP_MIN_ROWS rows (below it, cuBLAS and
    the SwiGLU kernel): both routes give the reference's rounding chain."""
    from helios_b200 import model as model_mod
    from helios_b200.config import Qwen3Config

    torch.manual_seed(5)
    cfg = Qwen3Config(vocab_size=64, context_length=4096, hidden_size=256, n_heads=2, n_layers=1, hidden_dim=512,
                      head_dim=128, n_kv_heads=1, dtype=torch.bfloat16)
    ff = model_mod.FeedForward(cfg).to(DEV)
    x = torch.randn(rows, 256, device=DEV).to(torch.bfloat16)
    with torch.inference_mode():
        default = ff(x)
        monkeypatch.setattr(model_mod, "FUSED_GATE_UP_MIN_ROWS", 1)
        fused = ff(x)
        monkeypatch.setattr(model_mod, "FUSED_GATE_UP_MIN_ROWS", 1 << 30)
        unfused = ff(x)
    torch.testing.assert_close(fused.float(), unfused.float(), rtol=2e-2, atol=2e-2)
    assert torch.equal(default, fused if rows >= model_mod.FUSED_GATE_UP_MIN_ROWS else unfused)
