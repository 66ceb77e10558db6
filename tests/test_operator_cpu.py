"""Operator renderer: an InferaDeployment CR renders to the golden
manifests; grace periods, RBAC, LWS, GAIE objects and status roll-up."""

import os

import pytest
import yaml

from infera_b200.operator.render import grace_seconds, render, rollup, to_yaml

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _cr():
    with open(os.path.join(GOLD, "operator_pd_k8s_cr.yaml")) as f:
        return yaml.safe_load(f)


def test_render_matches_golden():
    got = list(yaml.safe_load_all(to_yaml(render(_cr()))))
    with open(os.path.join(GOLD, "operator_pd_k8s_manifests.yaml")) as f:
        want = list(yaml.safe_load_all(f))
    assert got == want


def test_render_semantics():
    ms = render(_cr())
    kinds = [(m["kind"], m["metadata"]["name"]) for m in ms]
    assert ("LeaderWorkerSet", "llama70b-decode") in kinds and ("Deployment", "llama70b-prefill") in kinds
    assert ("InferencePool", "llama70b-pool") in kinds and ("HTTPRoute", "llama70b-route") in kinds
    assert kinds[0] == ("ServiceAccount", "llama70b-infera")
    pre = next(m for m in ms if m["metadata"]["name"] == "llama70b-prefill")
    pod = pre["spec"]["template"]["spec"]
    c = pod["containers"][0]
    assert pod["terminationGracePeriodSeconds"] == grace_seconds(90) == 155
    assert "--k8s-register" in c["command"] and "--disagg-mode" in c["command"]
    assert c["lifecycle"]["preStop"]["exec"]["command"] == ["sleep", "15"]
    assert pod["volumes"][0]["emptyDir"]["sizeLimit"] == "64Gi"
    dec = next(m for m in ms if m["metadata"]["name"] == "llama70b-decode")
    assert dec["spec"]["leaderWorkerTemplate"]["size"] == 2
    assert dec["spec"]["leaderWorkerTemplate"]["workerTemplate"]["spec"]["terminationGracePeriodSeconds"] == 120
    assert all(m["metadata"]["ownerReferences"][0]["uid"] == "1234" for m in ms)


def test_etcd_mode_and_errors():
    cr = _cr()
    cr["spec"]["discoveryBackend"] = "etcd"
    with pytest.raises(ValueError):
        render(cr)
    cr["spec"]["etcdEndpoint"] = "etcd:2379"
    cr["spec"]["gaie"]["enabled"] = False
    cr["spec"]["nats"] = {"deploy": True}
    ms = render(cr)
    assert not any(m["kind"] == "Role" for m in ms) and any(m["kind"] == "StatefulSet" for m in ms)
    w = next(m for m in ms if m["metadata"]["name"] == "llama70b-prefill")
    assert "--etcd-endpoint" in w["spec"]["template"]["spec"]["containers"][0]["command"]
    cr["spec"]["services"]["x"] = {"componentType": "bogus"}
    with pytest.raises(ValueError):
        render(cr)


def test_rollup():
    cr = _cr()
    st = rollup(cr, {"router": (2, 2), "prefill": (1, 1), "decode": (1, 0)})
    assert st["state"] == "Progressing" and st["services"]["decode"]["kind"] == "LeaderWorkerSet"
    st = rollup(cr, {"router": (2, 2), "prefill": (1, 1), "decode": (1, 1)})
    assert st["state"] == "Ready" and st["observedGeneration"] == 3
    assert rollup(cr, {"router": (0, 0)})["state"] == "Failed"
