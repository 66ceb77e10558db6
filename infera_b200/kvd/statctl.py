"""``python -m infera_b200.kvd.statctl --socket PATH [--json]``: print a
running kvd's counters (entries, bytes, L3 entries, gets / sets / hits /
misses / evictions, hit rate). Role of ``infera/kvd/statctl.py``."""

from __future__ import annotations

import argparse
import asyncio
import json


async def fetch(socket_path: str) -> dict:
    from infera_b200.kvd.client import KvdClient

    c = KvdClient(socket_path)
    await c.connect()
    try:
        st = await c.stats()
    finally:
        await c.close()
    d = {k: getattr(st, k) for k in st.__dataclass_fields__}
    lookups = d.get("hits_total", 0) + d.get("misses_total", 0)
    d["hit_rate"] = round(d.get("hits_total", 0) / lookups, 4) if lookups else None
    return d


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="python -m infera_b200.kvd.statctl")
    ap.add_argument("--socket", required=True)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    d = asyncio.run(fetch(a.socket))
    if a.json:
        print(json.dumps(d))
    else:
        for k, v in d.items():
            print(f"{k:>16}: {v}")


if __name__ == "__main__":
    main()
