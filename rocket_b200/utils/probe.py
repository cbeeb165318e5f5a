"""Mount probe ("test stand"): device and host facts, plus one trivial kernel
launch proving the sm_100a module loads.  Behavioural counterpart of the
reference's probe_mount / ignite (engines/glm5-moe-nvfp4-2b/src/engine.h:13-45)."""
from __future__ import annotations

import os
import platform


def _meminfo_kib(key: str):
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith(key + ":"):
                    return int(line.split()[1])
    except OSError:
        return None
    return None


def probe_mount(device: int = 0) -> dict:
    import torch
    facts = {
        "host": platform.node(),
        "kernel": platform.release(),
        "page_size": os.sysconf("SC_PAGE_SIZE"),
        "mem_available_kib": _meminfo_kib("MemAvailable"),
        "cuda_available": torch.cuda.is_available(),
    }
    if not torch.cuda.is_available():
        return facts
    p = torch.cuda.get_device_properties(device)
    free, total = torch.cuda.mem_get_info(device)
    facts.update({
        "gpu": p.name,
        "capability": f"{p.major}.{p.minor}",
        "sms": p.multi_processor_count,
        "gpu_total_bytes": total,
        "gpu_free_bytes": free,
        "gpu_count": torch.cuda.device_count(),
    })
    # ignite: one tiny kernel of ours (rmsnorm of a 1x64 row)
    from .. import ops
    x = torch.ones(1, 64, dtype=torch.bfloat16, device=f"cuda:{device}")
    y = ops.rmsnorm(x, torch.ones(64, dtype=torch.bfloat16, device=x.device), 1e-6)
    torch.cuda.synchronize(device)
    facts["ignite"] = bool(torch.allclose(y.float(), x.float()))
    # what this build of the kernel library supports
    facts["build"] = {"pdl": ops.pdl_supported(), "pdl_enabled": ops.pdl_enabled()}
    return facts
