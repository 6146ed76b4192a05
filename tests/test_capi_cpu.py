"""CPU checks of the C ABI: the library loads, exports every declared entry point, and
rejects bad arguments before touching a device (no GPU needed)."""
import ctypes
import os
import re

import pytest

from delta_phase_b200 import _capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "deltaphase_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"DP_API\s+[\w\s\*]*?\b(dp_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("dp_core_fwd", "dp_core_decode", "dp_laplace_fwd", "dp_ffn_fwd", "dp_gram",
              "dp_version", "dp_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    for s in declared_symbols():
        assert hasattr(lib, s), s
    assert set(declared_symbols()) == set(_capi.exported_symbols())


def test_version_and_status_strings():
    assert "sm_100a" in _capi.version()
    assert _capi.lib().dp_status_string(0) == b"ok"
    assert _capi.lib().dp_status_string(5) == b"device-side wait timed out"


def _core(**kw):
    a = dict(tk=None, tq=None, v=None, beta=None, in_dt=0, beta_dt=0, s_in=None, out=None,
             s_out=None, B=1, H=1, L=4, D=8, Dv=8, C=4, strides=None)
    a.update(kw)
    arr = (ctypes.c_int64 * 15)(*([0] * 15))
    return _capi.lib().dp_core_fwd(a["tk"], a["tq"], a["v"], a["beta"], a["in_dt"], a["beta_dt"],
                                   a["s_in"], a["out"], a["s_out"], a["B"], a["H"], a["L"], a["D"],
                                   a["Dv"], a["C"], arr if a["strides"] is None else a["strides"],
                                   None)


@pytest.mark.parametrize("kw,status", [
    (dict(B=-1), 1), (dict(C=0), 1), (dict(D=0), 1), (dict(D=129), 2), (dict(in_dt=9), 1),
    (dict(), 1),  # null pointers with B*H > 0
])
def test_core_argument_validation(kw, status):
    assert _core(**kw) == status
    assert _capi.lib().dp_last_error().decode().startswith("dp_core_fwd")


def test_core_empty_batch_is_a_no_op():
    assert _core(B=0) == 0


def test_other_entry_points_validate_arguments():
    L = _capi.lib()
    arr = (ctypes.c_int64 * 24)(*([0] * 24))
    assert L.dp_core_decode(None, None, None, None, None, None, 0, 0, None, 1, 1, 8, 8, arr, None) == 1
    assert L.dp_laplace_fwd(None, None, None, None, None, None, None, 0, 0, None, None, None,
                            1, 1, 4, 200, 8, 4, arr, None) == 2
    assert L.dp_gram(None, None, 0, 0, None, 1, 300, 8, None) == 2
    assert L.dp_ffn_fwd(None, 0, None, None, None, 4, 48, None, 0, None) == 2  # d not 2^k
    assert L.dp_ffn_fwd(None, 2, None, None, None, 4, 64, None, 0, None) == 1  # f16 x
    assert L.dp_ffn_workspace_size(10, 64, 1) >= 10 * 64 * 4 + 10 * 6 * 64 * 2


def test_block_glue_entry_points_validate_arguments():
    """dp_ln_conv_silu / dp_ln_conv_step / dp_layernorm reject bad sizes, dtypes and null
    pointers before touching the device; empty batches are no-ops."""
    L = _capi.lib()
    # kernel size above 8, float16 x, null pointers, negative sizes
    assert L.dp_ln_conv_silu(None, 0, None, None, 1e-5, None, None, None, 0, 1, 4, 64, 9, None) == 2
    assert L.dp_ln_conv_silu(None, 2, None, None, 1e-5, None, None, None, 0, 1, 4, 64, 4, None) == 1
    assert L.dp_ln_conv_silu(None, 0, None, None, 1e-5, None, None, None, 0, 1, 4, 64, 4, None) == 1
    assert L.dp_ln_conv_silu(None, 0, None, None, 1e-5, None, None, None, 0, 0, 4, 64, 4, None) == 0
    assert L.dp_ln_conv_step(None, 0, None, None, 1e-5, None, None, None, None, 0, -1, 64, 4, None) == 1
    assert L.dp_ln_conv_step(None, 0, None, None, 1e-5, None, None, None, None, 0, 2, 64, 4, None) == 1
    assert L.dp_ln_conv_step(None, 0, None, None, 1e-5, None, None, None, None, 0, 0, 64, 4, None) == 0
    assert L.dp_layernorm(None, 0, None, None, None, 1e-5, None, None, 2, 3, 64, None) == 1
    assert L.dp_layernorm(None, 0, None, None, None, 1e-5, None, None, 0, 3, 64, None) == 1
    assert L.dp_layernorm(None, 0, None, None, None, 1e-5, None, None, 0, 0, 64, None) == 0


def test_python_layer_rejects_cpu_tensors():
    import torch

    import delta_phase_b200 as dp
    x = torch.zeros(1, 1, 4, 8)
    with pytest.raises(RuntimeError):
        dp.delta_phase_chunkwise_fused(x, x, x, torch.zeros(1, 1, 4), 4)
    ffn = dp.LearnableSubstrateLerpFFN(16)
    with pytest.raises(RuntimeError):
        ffn(torch.zeros(3, 16))
