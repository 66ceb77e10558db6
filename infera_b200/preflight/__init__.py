"""Node preflight for a B200 box: host, GPU (NVML, read-only), NVLink
topology, GPU performance through this framework's kernels, KV-tier storage,
and a per-node JSON + combined HTML report. ``python -m infera_b200.preflight``.
Role of the reference's ``infera/tools/preflight``."""
