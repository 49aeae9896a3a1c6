"""Row kernels around the GEMMs vs the reference's formulas (oracle rounding points).

  * rmsnorm / add_rmsnorm: RMSNorm.forward (layers.py:36-40) after a bf16 residual add
    (layers.py:220-232); at most one bf16 ulp (fp32 reduction order, rsqrtf), hidden sizes
    covering every launch path (warp per row for 512..4096, CTA per row beyond);
  * gathered rmsnorm: the logit-row index_select + final norm (model.py:108-110);
  * swiglu: silu(gate) rounded to bf16, times up, rounded (layers.py:26-27);
  * embedding: exact row gather; ids outside the vocabulary are flagged, not read.
"""

import pytest
import torch
import torch.nn.functional as F

from helios_b200 import _native, ops
from oracle.numerics import rms_norm

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _ulps(a, b):
    return (a.contiguous().view(torch.int16).int() - b.contiguous().view(torch.int16).int()).abs()


@pytest.mark.parametrize("hidden", [512, 2560, 4096, 8192])
def test_add_rmsnorm_matches_reference_rounding(hidden):
    g = torch.Generator().manual_seed(hidden)
    rows = 300
    x = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    y = torch.randn(rows, hidden, generator=g).to(torch.bfloat16)
    scale = (0.5 + torch.rand(hidden, generator=g)).float()
    s_out = torch.empty(rows, hidden, dtype=torch.bfloat16, device=DEV)
    n_out = torch.empty_like(s_out)
    ops.add_rmsnorm(x.to(DEV), y.to(DEV), scale.to(DEV), 1e-6, s_out, n_out)
    ref_sum = x + y  # bf16 add: fp32 sum rounded once
    assert torch.equal(s_out.cpu(), ref_sum)
    u = _ulps(n_out.cpu(), rms_norm(ref_sum, scale, 1e-6))
    assert u.max().item() <= 1 and (u == 0).float().mean().item() > 0.98
    plain = ops.rmsnorm(x.to(DEV), scale.to(DEV), 1e-6)
    u = _ulps(plain.cpu(), rms_norm(x, scale, 1e-6))
    assert u.max().item() <= 1 and (u == 0).float().mean().item() > 0.98
    assert _native.device_status() == 0


def test_gathered_rmsnorm_is_index_select_then_norm():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(100, 2560, generator=g).to(torch.bfloat16)
    scale = torch.rand(2560, generator=g).float() + 0.5
    idx = torch.tensor([99, 0, 7, 7, 50])
    out = ops.rmsnorm(x.to(DEV), scale.to(DEV), 1e-6, row_index=idx.to(DEV))
    u = _ulps(out.cpu(), rms_norm(x[idx], scale, 1e-6))
    assert u.max().item() <= 1


def test_swiglu_matches_reference_rounding():
    g = torch.Generator().manual_seed(4)
    rows, inter = 257, 9728
    gate_up = (torch.randn(rows, 2 * inter, generator=g) * 2).to(torch.bfloat16)
    out = torch.empty(rows, inter, dtype=torch.bfloat16, device=DEV)
    ops.swiglu(gate_up.to(DEV), out)
    gate, up = gate_up[:, :inter], gate_up[:, inter:]
    ref = F.silu(gate.float()).to(torch.bfloat16) * up  # silu in fp32, rounded, then bf16 product
    u = _ulps(out.cpu(), ref)
    assert u.max().item() <= 1 and (u == 0).float().mean().item() > 0.99


def test_embedding_gathers_rows_and_flags_bad_ids():
    g = torch.Generator().manual_seed(5)
    table = torch.randn(1000, 512, generator=g).to(torch.bfloat16).to(DEV)
    ids = torch.tensor([3, 999, 0, 3], device=DEV)
    out = torch.empty(4, 512, dtype=torch.bfloat16, device=DEV)
    ops.embedding(ids, table, out)
    assert torch.equal(out, table[ids])
    _native.device_status(clear=True)
    ops.embedding(torch.tensor([1000, 2], device=DEV), table, out[:2])
    assert "token id outside the vocabulary" in _native.describe_status(_native.device_status(clear=True))
    assert torch.equal(out[1], table[2])
