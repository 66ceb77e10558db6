"""The benchmark's end-to-end fleet on CPU: etcd stand-in, router, worker
process attached to an in-process engine core, load generator - the tiny
model and trace, one rank."""

from infera_b200.bench.e2e import run_e2e_fleet
from infera_b200.common.net import free_tcp_port, free_tcp_port_block
from infera_b200.engine.llm_engine import EngineConfig, LLMEngine


def test_e2e_fleet_tiny(tmp_path):
    eng = LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=256), device="cpu")
    res = run_e2e_fleet(eng, model="tiny-dense", rank=0, world=1, barrier=lambda: None, sessions=range(0, 8),
                        rate=4.0, warmup_s=1.0, timed_s=4.0, seed=0, logdir=str(tmp_path), trace="tiny",
                        drain_s=5.0, appear_timeout=60,
                        ports={"etcd": free_tcp_port(), "router": free_tcp_port(), "worker0": free_tcp_port_block(1),
                               "events0": free_tcp_port_block(1)})
    assert res["errors"] == 0, res
    assert res["completed"] > 0
    assert res["iterations"] > 0 and len(res["ttfts"]) == res["completed"]
