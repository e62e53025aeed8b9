"""CPU-side checks of the C ABI: the library loads, exports every function
``include/nsm.h`` declares, and its pure host queries behave.  No kernel is
launched here (there is no GPU on the build machine)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def declared_functions() -> list[str]:
    text = (REPO / "include" / "nsm.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nsm_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from next_step_ai_b200 import _lib

    if not _lib.LIB_PATH.exists():
        from next_step_ai_b200.build import build

        build()
    return _lib.load()


def test_header_declares_the_bound_functions():
    from next_step_ai_b200 import _lib

    assert declared_functions() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(Path(lib._name)))
    for name in declared_functions():
        assert hasattr(raw, name), name


def test_status_strings_and_version(lib):
    from next_step_ai_b200 import _lib

    assert lib.nsm_abi_version() == _lib.ABI_VERSION == 4
    assert lib.nsm_status_string(0) == b"ok"
    assert lib.nsm_status_string(-5).startswith(b"workspace")
    assert lib.nsm_status_string(12345) == b"unknown status"


def test_static_array_holds_its_largest_call(lib):
    """nsm_decode_gathered_static keeps its scratch in a 6.5 MiB device array;
    the decode workspace layout at its limits (hidden 16384, 256 gathered
    blocks) must fit in it."""
    need = lib.nsm_decode_rows_workspace_bytes(16384, 256, 1)
    assert need == 6_423_296
    assert need <= 13 << 19


def test_workspace_size_queries(lib):
    b1 = lib.nsm_decode_workspace_bytes(16384, 53248, 208, 64)
    b0 = lib.nsm_decode_workspace_bytes(4096, 14336, 56, 64)
    assert b1 > b0 > 0
    assert b1 % 256 == 0
    assert lib.nsm_decode_workspace_bytes(0, 1, 1, 1) == 0
    assert lib.nsm_decode_rows_workspace_bytes(4096, 100, 4) > 0


def test_dropin_module_refuses_cpu_tensors():
    torch = pytest.importorskip("torch")
    from next_step_ai_b200 import triton_sparse_mlp as tsm

    x = torch.zeros((1, 64))
    with pytest.raises(RuntimeError, match="CUDA"):
        tsm.triton_sparse_input_linear_4bit(x, torch.zeros((1, 1), dtype=torch.int32),
                                            packed_weight=torch.zeros(32, dtype=torch.uint8),
                                            absmax=torch.ones(1), code=torch.zeros(16), out_features=1,
                                            in_features=64, quant_block_size=64, bias=None, block_size=32)
    with pytest.raises(RuntimeError, match="CUDA"):
        tsm.triton_sparse_mlp_decode_4bit_single_kernel_sm75(x, *([torch.zeros(1)] * 12), 64, 32, 64, 1)


def test_fused_composition_call_order(monkeypatch):
    """Same contract as the reference's tests/test_throughput_contract.py:364-407."""
    torch = pytest.importorskip("torch")
    from next_step_ai_b200 import triton_sparse_mlp as tsm

    calls = []

    def fake_output(x_flat, active_idx, flat_mask, **_):
        calls.append("output")
        return torch.ones_like(flat_mask, dtype=x_flat.dtype)

    def fake_input(x_flat, active_idx, **_):
        calls.append("input")
        assert tuple(x_flat.shape) == (1, 4) and tuple(active_idx.shape) == (1, 2)
        return torch.full((1, 3), 7.0, dtype=x_flat.dtype)

    monkeypatch.setattr(tsm, "triton_sparse_output_linear_4bit", fake_output)
    monkeypatch.setattr(tsm, "triton_sparse_input_linear_4bit", fake_input)
    e = torch.empty
    out = tsm.triton_fused_sparse_mlp_decode_4bit(
        torch.ones((1, 4), dtype=torch.float16), torch.tensor([[0, 1]], dtype=torch.int32),
        torch.ones((1, 4), dtype=torch.float16), gate_packed_weight=e(8, dtype=torch.uint8), gate_absmax=e(4),
        gate_code=e(16), gate_input_dim=4, gate_quant_block_size=64, gate_bias=None,
        up_packed_weight=e(8, dtype=torch.uint8), up_absmax=e(4), up_code=e(16), up_input_dim=4,
        up_quant_block_size=64, up_bias=None, down_packed_weight=e(8, dtype=torch.uint8), down_absmax=e(4),
        down_code=e(16), down_out_features=3, down_in_features=4, down_quant_block_size=64, down_bias=None,
        block_size=2)
    assert calls == ["output", "output", "input"]
    assert tuple(out.shape) == (1, 3)


def test_product_nf4_quantizer_matches_oracle():
    torch = pytest.importorskip("torch")
    import numpy as np

    from next_step_ai_b200.nf4 import nf4_code as t_code
    from next_step_ai_b200.nf4 import quantize_nf4 as t_quant
    from oracle.nf4 import nf4_code, quantize_nf4

    code = nf4_code()
    assert np.allclose(t_code().numpy(), code, atol=1e-7)
    w = (np.random.default_rng(5).standard_normal((64, 256)) * 0.02).astype(np.float32)
    p0, a0 = quantize_nf4(w, code)
    p1, a1 = t_quant(torch.from_numpy(w), torch.from_numpy(code))
    assert np.array_equal(p0, p1.numpy()) and np.array_equal(a0, a1.numpy())
