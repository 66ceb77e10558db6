"""``python -m infera_b200.operator render CR.yaml``: print the manifests."""

from __future__ import annotations

import sys

import yaml

from infera_b200.operator.render import render, to_yaml


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 2 or argv[0] != "render":
        raise SystemExit("usage: python -m infera_b200.operator render CR.yaml")
    with open(argv[1]) as f:
        cr = yaml.safe_load(f)
    sys.stdout.write(to_yaml(render(cr)))


if __name__ == "__main__":
    main()
