"""The engine on a B200 against the CPU oracle (plain full-sequence
forward on the same weights): eager and CUDA-graph decode, chunked prefill
and prefix-cache reuse."""

import pytest
import torch

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams
from infera_b200.models.reference import reference_greedy
from infera_b200.ops import kernels as K

pytestmark = pytest.mark.gpu


def _check(eng, prompts, outs, n):
    flips = 0
    for p, o in zip(prompts, outs):
        ref, margins = reference_greedy(eng.model, p, n)
        for i, (a, b) in enumerate(zip(o, ref)):
            if a != b:
                assert margins[i] < 0.15, (i, a, b, margins[i])
                flips += 1
                break
    return flips


@pytest.mark.parametrize("graphs", [False, True])
def test_engine_matches_oracle(graphs):
    cfg = EngineConfig(model="tiny-dense-gpu", num_pages=128, max_num_seqs=8, max_batched_tokens=96,
                       use_cuda_graphs=graphs)
    eng = LLMEngine(cfg, device="cuda:0")
    g = torch.Generator().manual_seed(0)
    prefix = torch.randint(0, 4096, (64,), generator=g).tolist()
    prompts = [torch.randint(0, 4096, (n,), generator=g).tolist() for n in (3, 130, 47)]
    prompts += [prefix + [1, 2, 3], prefix + [9, 8]]
    outs = eng.generate(prompts, SamplingParams(max_tokens=8, ignore_eos=True))
    torch.cuda.synchronize()
    assert K.scratch().read_status() == 0
    assert all(len(o) == 8 for o in outs)
    _check(eng, prompts, outs, 8)
    # second turn reuses the cached prefix + output
    p2 = prompts[1] + outs[1] + [5, 6, 7]
    before = eng.bm.stats["hit_tokens"]
    o2 = eng.generate([p2], SamplingParams(max_tokens=4, ignore_eos=True))[0]
    assert eng.bm.stats["hit_tokens"] - before >= 128
    _check(eng, [p2], [o2], 4)


def test_smoke_entry():
    from infera_b200.engine.smoke import run_smoke

    res = run_smoke("cuda:0")
    assert res["stats"]["finished"] == 3


def test_prefill_logits_match_oracle():
    from infera_b200.models.reference import reference_logits

    cfg = EngineConfig(model="tiny-dense-gpu", num_pages=64, max_num_seqs=4, max_batched_tokens=512,
                       use_cuda_graphs=False)
    eng = LLMEngine(cfg, device="cuda:0")
    g = torch.Generator().manual_seed(5)
    p = torch.randint(0, 4096, (300,), generator=g).tolist()
    eng.add_request("a", p, SamplingParams(max_tokens=1, ignore_eos=True))
    eng.step()
    got = eng.runner.last_logits[-1].float().cpu()
    ref = reference_logits(eng.model, p)[-1]
    rel = float((got - ref).norm() / ref.norm())
    assert rel < 2e-2, rel
