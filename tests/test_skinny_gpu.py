"""GPU checks of the decode-batch GEMM (dp_gemm_skinny) against a torch float32 matmul of
the same bf16 operands, and of the FFN's decode path built on it (dp_ffn_features between
two skinny GEMMs) against the fp64 oracle."""
import pytest
import torch

import delta_phase_b200 as dp
from delta_phase_b200 import _capi
from oracle import spectral as ospec

from helpers import TOL_BF16, rel_l2

pytestmark = pytest.mark.gpu

# fp32 accumulation of the same bf16 products in another order
TOL_SUM_ORDER = 1e-5


def _ref(x, w, bias, y0):
    r = x.float() @ w.float().t()
    if bias is not None:
        r = r + bias.float()
    return r if y0 is None else r + y0.float()


@pytest.mark.parametrize("M,N,K", [(16, 3088, 1024), (16, 1024, 6144), (1, 1024, 1024), (5, 33, 96),
                                   (16, 32000, 128), (3, 100, 32), (16, 9000, 224)])
@pytest.mark.parametrize("bias", [False, True])
def test_skinny_matches_matmul(M, N, K, bias):
    torch.manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    b = torch.randn(N, device="cuda").to(torch.bfloat16) if bias else None
    y = torch.empty(M, N, device="cuda")
    _capi.gemm_skinny(x, w, b, y)
    assert rel_l2(y, _ref(x, w, b, None)) < TOL_SUM_ORDER


def test_skinny_accumulate_strided_and_bf16_out():
    """A strided x (a column slice of a wider row), accumulation into a float32 y, and a
    bf16 y with a row stride wider than N."""
    torch.manual_seed(1)
    M, N, K = 16, 1024, 1024
    wide = torch.randn(M, 3 * K, device="cuda").to(torch.bfloat16)
    x = wide[:, K:2 * K]
    w = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    y0 = torch.randn(M, N, device="cuda")
    y = y0.clone()
    _capi.gemm_skinny(x, w, None, y, accumulate=True)
    _capi.gemm_skinny(x, w, None, y, accumulate=True)
    assert rel_l2(y, y0 + 2 * _ref(x, w, None, None)) < TOL_SUM_ORDER
    yb = torch.zeros(M, N + 64, device="cuda", dtype=torch.bfloat16)
    _capi.gemm_skinny(x, w, None, yb[:, :N])
    assert rel_l2(yb[:, :N].float(), _ref(x, w, None, None)) < TOL_BF16
    assert float(yb[:, N:].abs().max()) == 0.0   # nothing written past N


def test_skinny_deterministic():
    torch.manual_seed(2)
    x = torch.randn(16, 6144, device="cuda").to(torch.bfloat16)
    w = torch.randn(1024, 6144, device="cuda").to(torch.bfloat16)
    y1, y2 = torch.empty(16, 1024, device="cuda"), torch.empty(16, 1024, device="cuda")
    _capi.gemm_skinny(x, w, None, y1)
    _capi.gemm_skinny(x, w, None, y2)
    assert torch.equal(y1, y2)


def test_skinny_rejects_bad_shapes():
    x = torch.zeros(17, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(8, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="M must be <= 16"):
        _capi.gemm_skinny(x, w, None, torch.empty(17, 8, device="cuda"))
    x = torch.zeros(4, 48, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(8, 48, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        _capi.gemm_skinny(x, w, None, torch.empty(4, 8, device="cuda"))


@pytest.mark.parametrize("d,tokens", [(1024, 16), (256, 7), (128, 3)])
def test_ffn_decode_path(d, tokens):
    """LearnableSubstrateLerpFFN.add_to on a decode batch (bf16, <= 16 rows): DCT GEMM and
    folded combine on dp_gemm_skinny, dp_ffn_features between; against the oracle and
    against the cuBLAS path (dp_ffn_fwd_residual) on the same rows."""
    torch.manual_seed(d + tokens)
    ffn = dp.LearnableSubstrateLerpFFN(d, 4).cuda()
    with torch.no_grad():
        for n, p in ffn.named_parameters():
            p.copy_(torch.randn_like(p) * (1.0 if n == "substrate_logits" else 0.02))
    x = torch.randn(tokens, d, device="cuda").to(torch.bfloat16)
    r0 = torch.randn(tokens, d, device="cuda")
    r = r0.clone()
    with torch.no_grad():
        ffn.add_to(r, x)
    params = {k: v.detach().cpu().numpy() for k, v in ffn.state_dict().items()}
    ref = ospec.lerp_ffn(x.float().cpu().numpy(), params)
    assert rel_l2(r - r0, ref) < TOL_BF16
    Fm, dct = ffn.folded(torch.bfloat16)
    rc = r0.clone()
    ws = torch.empty(_capi.ffn_workspace_size(tokens, d, torch.bfloat16), device="cuda", dtype=torch.uint8)
    _capi.ffn_fwd_residual(x, dct, Fm, rc, ws)
    assert rel_l2(r - r0, rc - r0) < 1e-3
