"""Engine phase ranges in a profile: with ``trace_phases`` on (what the
engine's /start_profile sets), every step shows up in the torch profiler's
trace as named schedule / forward ranges; off, nothing is recorded."""

import torch

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams


def _names(prof):
    return {e.name for e in prof.events()}


def test_phase_ranges_in_profile():
    eng = LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=64), device="cpu")
    eng.trace_phases = True
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
        eng.generate([[1, 2, 3, 4, 5]], SamplingParams(max_tokens=3, ignore_eos=True))
    names = _names(prof)
    assert "schedule" in names
    assert any(n.startswith("forward prefill=1") for n in names)
    assert any(n.startswith("forward prefill=0 decode=1") for n in names)
    eng.trace_phases = False
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
        eng.generate([[7, 8, 9]], SamplingParams(max_tokens=2, ignore_eos=True))
    assert "schedule" not in _names(prof)
