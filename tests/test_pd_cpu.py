"""Prefill/decode disaggregation between two engines (tiny model, CPU; the
push uses the kernel wrapper's CPU path): the decode instance parks the
request, the prefill instance pushes the prompt's KV pages into the decode
instance's cache, and the decode output equals a single engine's."""

import torch

from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.request import SamplingParams


def _eng(**kw):
    return LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=128, **kw), device="cpu")


def _run_pair(prompt, n, room=77, dec=None, pre=None):
    dec = dec or _eng(disagg_mode="decode", kv_push_endpoint=f"local://pd-test-{room}")
    pre = pre or _eng(disagg_mode="prefill")
    ep = dec.pd_rendezvous.endpoint
    dec.add_request(f"d{room}", prompt, SamplingParams(max_tokens=n, ignore_eos=True,
                                                       kv_transfer={"do_remote_prefill": True, "room": room}))
    pre.add_request(f"p{room}", prompt, SamplingParams(max_tokens=1, ignore_eos=True,
                                                       kv_transfer={"do_remote_decode": True, "room": room,
                                                                    "decode_kv_endpoint": ep}))
    out = []
    for _ in range(500):
        if pre.has_unfinished():
            pre.step()
        if dec.has_unfinished():
            for o in dec.step():
                out.extend(o.new_token_ids)
        if not dec.has_unfinished() and not pre.has_unfinished():
            break
    return out, dec, pre


def test_pd_push_matches_single_engine():
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, 1024, (77,), generator=g).tolist()
    ref = _eng().generate([prompt], SamplingParams(max_tokens=6, ignore_eos=True))[0]
    out, dec, pre = _run_pair(prompt, 6)
    assert out == ref
    assert pre.pd_agent.stats["pushes"] == 1 and pre.pd_agent.stats["pages"] == (77 - 1 + 15) // 16
    assert dec.pd_rendezvous.stats["done"] == 1
    # the decode instance computed only the last prompt token itself
    assert dec.counters["prompt_tokens"] == 1
    # a second turn on the same decode instance reuses its cached prefix:
    # only the pages beyond it are pushed
    prompt2 = prompt + ref + torch.randint(0, 1024, (40,), generator=g).tolist()
    ref2 = _eng().generate([prompt2], SamplingParams(max_tokens=4, ignore_eos=True))[0]
    out2, dec, pre = _run_pair(prompt2, 4, room=78, dec=dec, pre=pre)
    assert out2 == ref2
    assert pre.pd_agent.stats["pages"] < (77 - 1 + 15) // 16 + (len(prompt2) - 1 + 15) // 16


def test_pd_push_timeout_falls_back_to_local_prefill():
    dec = _eng(disagg_mode="decode", kv_push_endpoint="local://pd-test-timeout")
    dec.pd_rendezvous.timeout_s = 0.05
    g = torch.Generator().manual_seed(6)
    prompt = torch.randint(0, 1024, (40,), generator=g).tolist()
    ref = _eng().generate([prompt], SamplingParams(max_tokens=3, ignore_eos=True))[0]
    dec.add_request("d", prompt, SamplingParams(max_tokens=3, ignore_eos=True,
                                                kv_transfer={"do_remote_prefill": True, "room": 9}))
    out = []
    while dec.has_unfinished():
        for o in dec.step():
            out.extend(o.new_token_ids)
    assert out == ref and dec.pd_rendezvous.stats["timeouts"] == 1


def test_pd_layerwise_push_inside_the_last_prefill_forward():
    import time

    g = torch.Generator().manual_seed(8)
    prompt = torch.randint(0, 1024, (70,), generator=g).tolist()
    ref = _eng().generate([prompt], SamplingParams(max_tokens=5, ignore_eos=True))[0]
    dec = _eng(disagg_mode="decode", kv_push_endpoint="local://pd-test-layerwise")
    pre = _eng(disagg_mode="prefill", max_batched_tokens=24)  # the prompt takes several chunks
    dec.add_request("d", prompt, SamplingParams(max_tokens=5, ignore_eos=True,
                                                kv_transfer={"do_remote_prefill": True, "room": 31}))
    dec.step()  # parks the request and publishes its pages
    pre.add_request("p", prompt, SamplingParams(max_tokens=1, ignore_eos=True,
                                                kv_transfer={"do_remote_decode": True, "room": 31,
                                                             "decode_kv_endpoint": dec.pd_rendezvous.endpoint}))
    out = []
    for _ in range(500):
        if pre.has_unfinished():
            pre.step()
            time.sleep(0.01)  # lets the agent thread resolve the page list between chunks
        if dec.has_unfinished():
            for o in dec.step():
                out.extend(o.new_token_ids)
        if not dec.has_unfinished() and not pre.has_unfinished():
            break
    assert out == ref
    assert pre.pd_agent.stats["layerwise"] == 1 and pre.pd_agent.stats["pushes"] == 1
    assert dec.counters["prompt_tokens"] == 1
