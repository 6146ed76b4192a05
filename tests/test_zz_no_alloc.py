"""The allocation-free FFN entry point (dp_ffn_fwd_noalloc), called through the C ABI.

It exists for callers that cannot allocate device memory where they run the FFN (a
stream being captured into a CUDA graph, runtimes whose allocator owns the device heap,
decode loops that must not block on the allocator): it takes its scratch from a fixed
array in the library instead of a caller workspace.  This file is collected last so a
run that stops at the first failure has already run every other test; it passes on its
own in a fresh process as well.
"""
import pytest
import torch

from delta_phase_b200 import LearnableSubstrateLerpFFN, _capi

from helpers import TOL_BF16, TOL_F32, rel_l2

pytestmark = pytest.mark.gpu


def _ffn(d, nb, seed):
    torch.manual_seed(seed)
    ffn = LearnableSubstrateLerpFFN(d, nb).cuda()
    with torch.no_grad():
        for n, p in ffn.named_parameters():
            p.copy_(torch.randn_like(p) * (1.0 if n == "substrate_logits" else 0.02))
    return ffn


def _workspace_ref(x, dct, F):
    """Output of the existing entry point dp_ffn_fwd (caller-provided workspace)."""
    y = torch.empty_like(x)
    ws = torch.empty(_capi.ffn_workspace_size(x.shape[0], x.shape[1], x.dtype), device=x.device,
                     dtype=torch.uint8)
    _capi.ffn_fwd(x, dct, F, y, ws)
    return y


@pytest.mark.parametrize("dtype,d,tokens,tol", [(torch.float32, 256, 100, TOL_F32),
                                                (torch.bfloat16, 1024, 300, TOL_BF16),
                                                (torch.float32, 64, 7, TOL_F32)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, d, tokens, tol):
    ffn = _ffn(d, 4, 3)
    F, dct = ffn.folded(dtype)
    for call in range(2):  # two calls in a row share (and overwrite) the static scratch
        x = torch.randn(tokens, d, device="cuda").to(dtype)
        ref = _workspace_ref(x, dct, F)
        y = torch.empty_like(x)
        _capi.ffn_fwd_noalloc(x, dct, F, y)
        torch.cuda.synchronize()
        assert rel_l2(y.float(), ref.float()) < tol, call


def test_noalloc_rejects_sizes_beyond_its_scratch():
    d = 1024
    limit = _capi.ffn_noalloc_max_tokens(d, torch.bfloat16)
    assert 0 < limit < 4096
    x = torch.zeros(limit + 1, d, device="cuda", dtype=torch.bfloat16)
    F = torch.zeros(6 * d, d, device="cuda", dtype=torch.bfloat16)
    dct = torch.zeros(d, d, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_capi.DeltaPhaseCudaError, match="static scratch"):
        _capi.ffn_fwd_noalloc(x, dct, F, torch.empty_like(x))


@pytest.mark.parametrize("dtype,d,tol", [(torch.bfloat16, 1024, TOL_BF16), (torch.float32, 4096, TOL_F32)])
def test_noalloc_at_its_token_limit(dtype, d, tol):
    """Exactly dp_ffn_noalloc_max_tokens tokens: the largest call, where the features
    (placed after the DCT projections at the next 256-byte boundary) reach closest to the
    end of the fixed scratch."""
    ffn = _ffn(d, 2, 5)
    F, dct = ffn.folded(dtype)
    tokens = _capi.ffn_noalloc_max_tokens(d, dtype)
    for _ in range(2):
        x = torch.randn(tokens, d, device="cuda").to(dtype)
        ref = _workspace_ref(x, dct, F)
        y = torch.empty_like(x)
        _capi.ffn_fwd_noalloc(x, dct, F, y)
        torch.cuda.synchronize()
        assert rel_l2(y.float(), ref.float()) < tol
