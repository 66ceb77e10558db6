"""``python -m infera_b200.preflight [--host] [--gpu] [--topology] [--perf]
[--storage] [--storage-path DIR] [--storage-mib N] [--dump-path DIR]``

With no probe flag every probe runs. Writes ``<dump>/<hostname>.json`` and
renders ``<dump>/infera_preflight_report.html`` over every node JSON in the
dump directory (several nodes writing to one shared directory get one
combined report, with cross-node consistency findings). Exit code 1 when
any finding is ``fail``.
"""

from __future__ import annotations

import argparse
import glob
import html
import json
import os
import platform
import sys

from infera_b200.preflight import checks
from infera_b200.preflight.checks import LEVELS, Finding


def run(args) -> dict:
    want = {k: getattr(args, k) for k in ("host", "gpu", "topology", "perf", "storage")}
    every = not any(want.values())
    report: dict = {"node": platform.node(), "findings": []}

    def take(name, res):
        data, fs = res
        report[name] = data
        report["findings"].extend(x.to_dict() for x in fs)

    if every or want["host"]:
        take("host", checks.host_info())
    if every or want["gpu"]:
        take("gpu", checks.gpu_info())
    if every or want["topology"]:
        take("topology", checks.gpu_topology())
    if every or want["perf"]:
        take("perf", checks.gpu_perf(gemm_n=args.gemm_n, iters=args.iters))
    if every or want["storage"]:
        take("storage", checks.storage(args.storage_path, mib=args.storage_mib))
    report["level"] = max((f["level"] for f in report["findings"]), key=lambda x: LEVELS[x], default="info")
    return report


def render_html(nodes: dict[str, dict], cross: list[Finding]) -> str:
    rows = []
    for node, r in sorted(nodes.items()):
        for f in r.get("findings", []):
            rows.append((node, f["level"], f["check"], f["message"]))
    for f in cross:
        rows.append(("(all nodes)", f.level, f.check, f.message))
    color = {"info": "#e8f4e8", "warn": "#fff4d6", "fail": "#fbdada"}
    body = "\n".join(f"<tr style='background:{color.get(lv, '#fff')}'><td>{html.escape(n)}</td><td>{lv}</td>"
                     f"<td>{html.escape(c)}</td><td>{html.escape(m)}</td></tr>" for n, lv, c, m in rows)
    summary = "".join(f"<li>{html.escape(n)}: <b>{r.get('level', 'info')}</b></li>" for n, r in sorted(nodes.items()))
    return ("<!doctype html><html><head><meta charset='utf-8'><title>infera-b200 preflight</title></head><body>"
            f"<h1>Preflight</h1><ul>{summary}</ul><table border='1' cellpadding='4'>"
            f"<tr><th>node</th><th>level</th><th>check</th><th>finding</th></tr>{body}</table></body></html>")


def write_report(dump: str, report: dict) -> tuple[str, list[Finding]]:
    os.makedirs(dump, exist_ok=True)
    with open(os.path.join(dump, f"{report['node']}.json"), "w") as fh:
        json.dump(report, fh, indent=1, default=str)
    nodes = {}
    for p in glob.glob(os.path.join(dump, "*.json")):
        try:
            with open(p) as fh:
                r = json.load(fh)
            nodes[r.get("node", os.path.basename(p))] = r
        except (OSError, ValueError):
            continue
    cross = checks.consistency(nodes) if len(nodes) > 1 else []
    out = os.path.join(dump, "infera_preflight_report.html")
    with open(out, "w") as fh:
        fh.write(render_html(nodes, cross))
    return out, cross


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="python -m infera_b200.preflight")
    for k in ("host", "gpu", "topology", "perf", "storage"):
        ap.add_argument(f"--{k}", action="store_true")
    ap.add_argument("--storage-path", default=os.environ.get("INFERA_PREFLIGHT_STORAGE_PATH", "/tmp/infera-kv"))
    ap.add_argument("--storage-mib", type=int, default=int(os.environ.get("INFERA_PREFLIGHT_STORAGE_MIB", "1024")))
    ap.add_argument("--gemm-n", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--dump-path", default="output/preflight")
    args = ap.parse_args(argv)
    report = run(args)
    path, cross = write_report(args.dump_path, report)
    for f in report["findings"]:
        print(f"[{f['level']:4s}] {f['check']}: {f['message']}")
    for f in cross:
        print(f"[{f.level:4s}] {f.check}: {f.message}")
    print(f"report: {path}")
    sys.exit(1 if report["level"] == "fail" or any(f.level == "fail" for f in cross) else 0)
