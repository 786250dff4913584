"""Environment report (``scripts/diagnose.py`` of the reference): ``python -m verl_omni_b200.cli.diagnose``."""

from __future__ import annotations

import json
import os
import platform
import subprocess
import sys


def collect() -> dict:
    info = {"python": sys.version.split()[0], "platform": platform.platform()}
    try:
        import torch

        info["torch"] = torch.__version__
        info["cuda_available"] = torch.cuda.is_available()
        info["torch_cuda"] = torch.version.cuda
        info["nccl"] = ".".join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else None
        if torch.cuda.is_available():
            info["devices"] = [{"name": torch.cuda.get_device_name(i),
                                "capability": ".".join(map(str, torch.cuda.get_device_capability(i))),
                                "memory_gb": round(torch.cuda.get_device_properties(i).total_memory / 2**30, 1)}
                               for i in range(torch.cuda.device_count())]
    except Exception as e:  # noqa: BLE001
        info["torch_error"] = str(e)
    try:
        from verl_omni_b200.ops._ext import so_path

        info["extension"] = so_path()
    except Exception as e:  # noqa: BLE001
        info["extension_error"] = str(e)
    try:
        out = subprocess.run(["nvcc", "--version"], capture_output=True, text=True, timeout=20).stdout
        info["nvcc"] = out.strip().splitlines()[-1] if out else None
    except Exception:  # noqa: BLE001
        info["nvcc"] = None
    info["env"] = {k: v for k, v in os.environ.items() if k.startswith(("VO_", "VERL_", "NCCL_", "CUDA_VISIBLE"))}
    return info


if __name__ == "__main__":
    print(json.dumps(collect(), indent=2))
