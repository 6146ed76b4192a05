"""GPU parity of the spectral Lerp FFN (dp_ffn_fold + dp_ffn_fwd) and of the drop-in
block forward/step against golden vectors from the reference and the fp64 oracle."""
import numpy as np
import pytest
import torch

import delta_phase_b200 as dp
from oracle import spectral as ospec

from helpers import TOL_BF16, TOL_F32, load_golden, rel_l2, round_bf16, to_dev

pytestmark = pytest.mark.gpu


def _ffn_from_golden(g, i):
    p = f"c{i}_p_"
    params = {k[len(p):]: g[k] for k in g.files if k.startswith(p)}
    d = params["mat_dct"].shape[0]
    ffn = dp.LearnableSubstrateLerpFFN(d, num_banks=int(g[f"c{i}_nb"])).cuda()
    ffn.load_state_dict({k: torch.from_numpy(v).float() for k, v in params.items()})
    return ffn, params


def test_ffn_golden_fp32():
    g = load_golden("ffn")
    for i in range(int(g["n_cases"])):
        ffn, _ = _ffn_from_golden(g, i)
        with torch.no_grad():
            y = ffn(to_dev(g[f"c{i}_x"].astype(np.float32)))
        assert rel_l2(y, g[f"c{i}_y"]) < TOL_F32, i


def test_ffn_config4_bf16_slice():
    """d_model = 1024, nb = 4, bf16 activations, params ~ N(0, 0.02), router ~ N(0, 1)."""
    torch.manual_seed(0)
    d, nb, tokens = 1024, 4, 512
    ffn = dp.LearnableSubstrateLerpFFN(d, nb).cuda()
    with torch.no_grad():
        for n, p in ffn.named_parameters():
            p.copy_(torch.randn_like(p) * (1.0 if n == "substrate_logits" else 0.02))
    x = torch.randn(tokens, d, device="cuda").to(torch.bfloat16)
    with torch.no_grad():
        y = ffn(x)
    assert y.dtype == torch.bfloat16
    params = {k: v.detach().cpu().numpy() for k, v in ffn.state_dict().items()}
    ref = ospec.lerp_ffn(x.float().cpu().numpy(), params)
    assert rel_l2(y.float(), ref) < TOL_BF16


def test_ffn_refolds_after_parameter_update():
    g = load_golden("ffn")
    ffn, params = _ffn_from_golden(g, 0)
    x = to_dev(g["c0_x"].astype(np.float32))
    with torch.no_grad():
        ffn(x)
        ffn.substrate_logits.add_(0.5)
        y = ffn(x)
    params = {k: v.detach().cpu().numpy() for k, v in ffn.state_dict().items()}
    assert rel_l2(y, ospec.lerp_ffn(g["c0_x"], params)) < TOL_F32


def _block_from_golden(g, i):
    p = f"c{i}_"
    params = {k[len(p) + 2:]: g[k] for k in g.files if k.startswith(p + "p_")}
    blk = dp.DeltaPhaseHolographicBlock(d_model=64, n_heads=4, chunk_size=int(g[p + "C"]),
                                        beta_mode=str(g[p + "beta_mode"])).cuda().eval()
    blk.load_state_dict({k: torch.from_numpy(v).float() for k, v in params.items()})
    return blk


def test_block_forward_and_step_golden():
    g = load_golden("block")
    for i in range(int(g["n_cases"])):
        p = f"c{i}_"
        blk = _block_from_golden(g, i)
        x = to_dev(g[p + "x"].astype(np.float32))
        with torch.no_grad():
            out, M = blk(x)
            st = None
            outs = []
            for t in range(x.shape[1]):
                o, st = blk.step(x[:, t:t + 1], st)
                outs.append(o)
        assert rel_l2(out, g[p + "out"]) < TOL_F32, i
        assert rel_l2(M, g[p + "M"]) < TOL_F32, i
        assert rel_l2(torch.cat(outs, 1), g[p + "out_step"]) < TOL_F32, i
        assert rel_l2(st[1], g[p + "M_step"]) < TOL_F32, i
        assert blk.last_beta.shape[:2] == (2, 4)


def test_block_bf16_autocast_runs():
    g = load_golden("block")
    blk = _block_from_golden(g, 0)
    x = to_dev(g["c0_x"].astype(np.float32))
    with torch.no_grad():
        ref, _ = blk(x)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out, M = blk(x)
    assert torch.isfinite(out.float()).all()
    assert rel_l2(out.float(), ref) < 5e-2


def test_model_prefill_then_decode():
    cfg = dp.DeltaPhaseConfig(dim=128, n_heads=2, n_layers=2, vocab_size=500, chunk_size=32)
    torch.manual_seed(0)
    model = dp.DeltaPhaseModel(cfg).cuda().eval()
    ids = torch.randint(0, 500, (2, 40), device="cuda")
    with torch.no_grad():
        logits = model(ids)
        st = None
        for t in range(40):
            lt, st = model.step(ids[:, t:t + 1], st)
    assert logits.shape == (2, 40, 500)
    assert rel_l2(lt[:, 0], logits[:, -1]) < TOL_F32


@pytest.mark.parametrize("d", [64, 128, 256, 512, 1024, 2048])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tokens", [77, 700])
def test_ffn_widths(d, dtype, tokens):
    """Every width of the warp feature kernels (256..1024: three warps per token up to 512
    tokens, one warp per token above) and of the block-per-token one (64, 128, 2048),
    float32 and bf16 activations, against the fp64 oracle."""
    torch.manual_seed(d)
    nb = 4
    ffn = dp.LearnableSubstrateLerpFFN(d, nb).cuda()
    with torch.no_grad():
        for n, p in ffn.named_parameters():
            p.copy_(torch.randn_like(p) * (1.0 if n == "substrate_logits" else 0.02))
    x = torch.randn(tokens, d, device="cuda").to(dtype)
    with torch.no_grad():
        y = ffn(x)
    params = {k: v.detach().cpu().numpy() for k, v in ffn.state_dict().items()}
    ref = ospec.lerp_ffn(x.float().cpu().numpy(), params)
    assert rel_l2(y.float(), ref) < (TOL_BF16 if dtype == torch.bfloat16 else TOL_F32)


@pytest.mark.parametrize("d,dtype", [(1024, torch.bfloat16), (256, torch.float32), (64, torch.bfloat16)])
def test_ffn_residual_accumulate(d, dtype):
    """dp_ffn_fwd_residual (through LearnableSubstrateLerpFFN.add_to): r += FFN(x) in
    float32, the block's x + ffn(norm2(x)) (layers.py:243, 290), against the fp64 oracle."""
    torch.manual_seed(d + 1)
    nb, tokens = 4, 16
    ffn = dp.LearnableSubstrateLerpFFN(d, nb).cuda()
    with torch.no_grad():
        for n, p in ffn.named_parameters():
            p.copy_(torch.randn_like(p) * (1.0 if n == "substrate_logits" else 0.02))
    x = torch.randn(tokens, d, device="cuda").to(dtype)
    r0 = torch.randn(tokens, d, device="cuda")
    r = r0.clone()
    with torch.no_grad():
        out = ffn.add_to(r, x)
    assert out.data_ptr() == r.data_ptr()
    params = {k: v.detach().cpu().numpy() for k, v in ffn.state_dict().items()}
    ref = ospec.lerp_ffn(x.float().cpu().numpy(), params)
    tol = TOL_BF16 if dtype == torch.bfloat16 else TOL_F32
    assert rel_l2(r - r0, ref) < tol


def test_ffn_unaligned_rows():
    """x starting 2 bytes past a 16-byte boundary takes the block-per-token kernel."""
    torch.manual_seed(3)
    d, nb, tokens = 256, 4, 40
    ffn = dp.LearnableSubstrateLerpFFN(d, nb).cuda()
    with torch.no_grad():
        for n, p in ffn.named_parameters():
            p.copy_(torch.randn_like(p) * (1.0 if n == "substrate_logits" else 0.02))
    buf = torch.randn(tokens * d + 1, device="cuda").to(torch.bfloat16)
    x = buf[1:].view(tokens, d)
    with torch.no_grad():
        y = ffn(x)
    params = {k: v.detach().cpu().numpy() for k, v in ffn.state_dict().items()}
    ref = ospec.lerp_ffn(x.float().cpu().numpy(), params)
    assert rel_l2(y.float(), ref) < TOL_BF16


def test_ffn_follows_bf16_autocast():
    """float32 activations under bf16 autocast (the LayerNorm in front of the FFN returns
    float32) take the bf16 path, as the reference's matmuls would, and return bf16."""
    torch.manual_seed(7)
    d, nb, tokens = 1024, 4, 64
    ffn = dp.LearnableSubstrateLerpFFN(d, nb).cuda()
    with torch.no_grad():
        for n, p in ffn.named_parameters():
            p.copy_(torch.randn_like(p) * (1.0 if n == "substrate_logits" else 0.02))
    x = torch.randn(tokens, d, device="cuda")
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = ffn(x)
    assert y.dtype == torch.bfloat16
    params = {k: v.detach().cpu().numpy() for k, v in ffn.state_dict().items()}
    ref = ospec.lerp_ffn(x.to(torch.bfloat16).float().cpu().numpy(), params)
    assert rel_l2(y.float(), ref) < TOL_BF16


@pytest.mark.parametrize("L,d,out_dtype", [(37, 256, torch.float32), (70, 1024, torch.bfloat16), (5, 64, torch.float32),
                                           (100, 512, torch.float32), (2, 768, torch.bfloat16), (33, 320, torch.float32)])
def test_ln_conv_silu_kernel(L, d, out_dtype):
    """dp_ln_conv_silu against torch's LayerNorm -> causal depthwise conv -> SiLU ->
    residual (tile edges, the first k-1 tokens' zero padding, several sequences; d = 256 j
    on the statistics-then-channels kernel, other widths on the staged one)."""
    from delta_phase_b200 import _capi
    torch.manual_seed(L)
    B = 3
    norm = torch.nn.LayerNorm(d).cuda()
    conv = dp.ShortCausalConv1D(d).cuda()
    with torch.no_grad():
        norm.weight.uniform_(0.5, 1.5)
        norm.bias.uniform_(-0.2, 0.2)
        x = torch.randn(B, L, d, device="cuda") * 2 + 0.3
        ref = conv(norm(x))
        out = torch.empty(B, L, d, device="cuda", dtype=out_dtype)
        _capi.ln_conv_silu(x, norm.weight, norm.bias, norm.eps, conv.conv.weight.reshape(d, -1).contiguous(),
                           conv.conv.bias, out)
    tol = 1e-5 if out_dtype == torch.float32 else 4e-3
    assert rel_l2(out.float(), ref) < tol


@pytest.mark.parametrize("x_dtype,y_dtype,resid", [(torch.float32, torch.float32, False),
                                                   (torch.bfloat16, torch.bfloat16, True),
                                                   (torch.float32, torch.bfloat16, True)])
def test_layernorm_kernel(x_dtype, y_dtype, resid):
    from delta_phase_b200 import _capi
    torch.manual_seed(1)
    rows, d = 300, 1024
    norm = torch.nn.LayerNorm(d).cuda()
    with torch.no_grad():
        norm.weight.uniform_(0.5, 1.5)
        norm.bias.uniform_(-0.2, 0.2)
        x = (torch.randn(rows, d, device="cuda") * 3).to(x_dtype)
        r = torch.randn(rows, d, device="cuda") if resid else None
        s_ref = x.float() + (r if resid else 0)
        y = torch.empty(rows, d, device="cuda", dtype=y_dtype)
        s = torch.empty(rows, d, device="cuda") if resid else None
        _capi.layernorm(x, norm.weight, norm.bias, norm.eps, y, residual=r, sum_out=s)
        ref = norm(s_ref)
    assert rel_l2(y.float(), ref) < (1e-5 if y_dtype == torch.float32 else 4e-3)
    if resid:
        assert rel_l2(s, s_ref) < 1e-7


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [512, 1024, 320])
def test_ln_conv_step_kernel(out_dtype, d):
    """dp_ln_conv_step over 6 tokens against LayerNorm + ShortCausalConv1D.step, the
    (B, d, k-1) conv state carried through the kernel (d = 256 j on the register-resident
    kernel, others on the general one)."""
    from delta_phase_b200 import _capi
    torch.manual_seed(4)
    B = 5
    norm = torch.nn.LayerNorm(d).cuda()
    conv = dp.ShortCausalConv1D(d).cuda()
    with torch.no_grad():
        norm.weight.uniform_(0.5, 1.5)
        norm.bias.uniform_(-0.2, 0.2)
        st_ref = torch.randn(B, d, 3, device="cuda")
        st = st_ref.clone()
        for _ in range(6):
            x = torch.randn(B, 1, d, device="cuda") * 2
            ref, st_ref = conv.step(norm(x), conv_state=st_ref)
            out = torch.empty(B, d, device="cuda", dtype=out_dtype)
            _capi.ln_conv_step(x.view(B, d), norm.weight, norm.bias, norm.eps,
                               conv.conv.weight.reshape(d, -1).contiguous(), conv.conv.bias, st, out)
            assert rel_l2(out.float(), ref.view(B, d)) < (1e-5 if out_dtype == torch.float32 else 4e-3)
            assert rel_l2(st, st_ref) < 1e-6
