"""Weight-streaming GEMM (hb_stream_gemm) for decode-tick row counts.

Replaces the nn.Linear projections (src/helios/runtime/qwen3/layers.py:26-27, :131-146) at
m <= 256 token rows. Checked against an fp32 product of the same bf16 operands (both
accumulate in fp32; only the summation order differs, so the bf16 outputs agree to within
a bf16 rounding step), for the Qwen3-4B projection shapes and odd sizes; two calls give
identical bits (split weight tiles add their parts in a fixed order), and the tile counters
in the workspace are back at zero after every call.
"""

import pytest
import torch

from helios_b200 import _native, ops

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")

CASES = [
    (1, 256, 128),        # one token, two weight tiles
    (33, 2560, 4096),     # o-proj, 32 decode rows + a drafted row
    (128, 6144, 2560),    # q|k|v at config 4
    (128, 2560, 9728),    # down at config 4
    (256, 19456, 2560),   # gate|up at the row limit
    (77, 1024, 640),      # odd sizes
]


def _ref(x, w):
    return x.float() @ w.float().T


@pytest.mark.parametrize("m,n,k", CASES)
def test_stream_gemm_matches_fp32_product(m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=DEV, generator=g) / k ** 0.5).to(torch.bfloat16)
    got = ops.stream_gemm(x, w)
    want = _ref(x, w)
    err = (got.float() - want).abs()
    # bf16 output rounding (2^-9 relative) plus fp32 order differences
    bound = want.abs() * 2.0 ** -8 + 1e-3
    assert bool((err <= bound).all()), float((err / bound).max())
    again = ops.stream_gemm(x, w)
    assert torch.equal(got, again)
    nbytes = int(_native.load().hb_stream_gemm_workspace_bytes(m, n, k))
    counters = ops._STREAM_WS[DEV][: (n // 128) * 4].view(torch.int32)
    assert int(counters.abs().sum()) == 0 and nbytes > 0
    assert _native.device_status() == 0


def test_stream_gemm_rejects_unsupported_sizes():
    x = torch.zeros(300, 128, device=DEV, dtype=torch.bfloat16)
    w = torch.zeros(256, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.stream_gemm(x, w)  # more than 256 rows
    with pytest.raises(ValueError):
        ops.stream_gemm(x[:8], torch.zeros(200, 128, device=DEV, dtype=torch.bfloat16))  # n % 128
