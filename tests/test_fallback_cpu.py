"""CPU: the 16-bit -> fp32 overflow guard's control flow (the reference recomputes in fp32 when an
fp16 pass overflows, model.py:179-193) and the tracing helper; no kernel runs here."""

import torch

from boltz_mlx_b200.triangle_attention import TriangleAttention, nvtx_range, run_with_fp32_fallback


def test_fallback_runs_fp32_only_on_nonfinite_output():
    calls = []

    def run16():
        calls.append("16")
        return torch.tensor([1.0, float("inf")])

    def run32():
        calls.append("32")
        return torch.tensor([1.0, 2.0])

    out, fell = run_with_fp32_fallback(run16, run32, lambda t: bool(torch.isfinite(t).all()))
    assert fell and calls == ["16", "32"] and torch.equal(out, torch.tensor([1.0, 2.0]))
    calls.clear()
    out, fell = run_with_fp32_fallback(lambda: (calls.append("16"), torch.ones(3))[1], run32,
                                       lambda t: bool(torch.isfinite(t).all()))
    assert not fell and calls == ["16"] and torch.equal(out, torch.ones(3))
    out, fell = run_with_fp32_fallback(lambda: torch.tensor([float("nan")]), run32,
                                       lambda t: bool(torch.isfinite(t).all()))
    assert fell


def test_fallback_is_off_by_default_and_counts_events():
    mod = TriangleAttention(precision="bf16")
    assert mod.fp32_fallback is False and mod.nonfinite_events == 0


def test_nvtx_range_is_a_context_manager():
    with nvtx_range("triattn.test"):
        pass
