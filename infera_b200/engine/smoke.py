"""One tiny decode of the flagship dense model architecture on a GPU.

Runs the real kernels (tcgen05 GEMM, paged prefill FA, split-KV decode,
fused norms / RoPE, sampling) through the engine on a 2-layer model of the
Llama-3.1-8B layer shape, and checks the kernel status word.
"""

from __future__ import annotations

import torch


def run_smoke(device: str = "cuda:0") -> dict:
    from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
    from infera_b200.engine.request import SamplingParams
    from infera_b200.ops import kernels as K

    cfg = EngineConfig(model="llama-3.1-8b", num_pages=256, max_num_seqs=8, max_batched_tokens=512,
                       use_cuda_graphs=True, model_overrides={"num_layers": 2, "max_model_len": 4096})
    eng = LLMEngine(cfg, device=device)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 128000, (n,), generator=g).tolist() for n in (37, 300, 16)]
    outs = eng.generate(prompts, SamplingParams(max_tokens=4, ignore_eos=True))
    torch.cuda.synchronize()
    status = K.scratch(torch.device(device)).read_status()
    if status != 0:
        raise RuntimeError(f"kernel status word {status}")
    assert all(len(o) == 4 for o in outs), outs
    return {"outputs": outs, "stats": eng.stats()}


if __name__ == "__main__":
    print(run_smoke())
