"""GPU architecture detection for the worker record and preflight checks.

Returns ``sm_<major><minor>`` of the current (or given) CUDA device, from
torch when a GPU is visible, else from ``nvidia-smi``'s compute capability,
else None. This framework's kernels are built for sm_100a only; other
architectures are reported, not served (role of ``infera/common/arch.py:49``,
which detects the reference's gfx targets).
"""

from __future__ import annotations

import shutil
import subprocess

SUPPORTED = ("sm_100",)


def gpu_arch(device: int = 0) -> str | None:
    try:
        import torch

        if torch.cuda.is_available():
            major, minor = torch.cuda.get_device_capability(device)
            return f"sm_{major}{minor}"
    except Exception:
        pass
    smi = shutil.which("nvidia-smi")
    if smi:
        try:
            out = subprocess.run([smi, "--query-gpu=compute_cap", "--format=csv,noheader", f"--id={device}"],
                                 stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, timeout=10, text=True)
            cap = out.stdout.strip().splitlines()[0].strip()
            major, _, minor = cap.partition(".")
            return f"sm_{int(major)}{int(minor or 0)}"
        except Exception:
            return None
    return None


def is_supported(arch: str | None) -> bool:
    return arch in SUPPORTED
