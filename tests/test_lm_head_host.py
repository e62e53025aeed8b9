"""Host side of the NF4 LM head (no GPU): quant block-size resolution as the
reference's ``_resolve_lm_head_nf4_quant_block_size`` and the no-fallback
rule (host tensors are refused)."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")
from next_step_ai_b200 import lm_head  # noqa: E402


def test_quant_block_size_resolution(monkeypatch):
    monkeypatch.delenv("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", raising=False)
    assert lm_head.resolve_lm_head_nf4_quant_block_size(16384) == 64
    assert lm_head.resolve_lm_head_nf4_quant_block_size(4096 + 128) == 64
    assert lm_head.resolve_lm_head_nf4_quant_block_size(96) == 32
    with pytest.raises(RuntimeError, match="Unable to select"):
        lm_head.resolve_lm_head_nf4_quant_block_size(100)
    monkeypatch.setenv("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", "256")
    assert lm_head.resolve_lm_head_nf4_quant_block_size(16384) == 256
    monkeypatch.setenv("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", "96")     # does not divide: ignored
    assert lm_head.resolve_lm_head_nf4_quant_block_size(16384) == 64
    monkeypatch.setenv("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", "x")
    assert lm_head.resolve_lm_head_nf4_quant_block_size(16384) == 64


def test_host_tensors_are_refused():
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        lm_head.Nf4LmHead(torch.zeros(64 * 512, dtype=torch.uint8), torch.zeros(512), torch.zeros(16),
                          out_features=64, in_features=1024)


def test_quant_block_size_matches_reference(monkeypatch):
    """The reference's _resolve_lm_head_nf4_quant_block_size on the same
    inputs when the fixture was made (tests/golden/make_golden.py)."""
    import json
    from pathlib import Path

    gold = json.loads((Path(__file__).parent / "golden" / "checkpoint.json").read_text())["lm_head_qbs"]
    assert len(gold) >= 8
    for c in gold:
        monkeypatch.delenv("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", raising=False)
        if c["env"] is not None:
            monkeypatch.setenv("STREAMING_GPU_LM_HEAD_NF4_BLOCK_SIZE", c["env"])
        if "error" in c:
            with pytest.raises(RuntimeError) as e:
                lm_head.resolve_lm_head_nf4_quant_block_size(c["in_features"])
            assert str(e.value) == c["error"]
        else:
            assert lm_head.resolve_lm_head_nf4_quant_block_size(c["in_features"]) == c["qbs"], c
