"""Hardware / software provenance recorded in every result JSON (the reference's
runner stamps each stage result with ``_hardware_provenance``,
``deepseek_v41/runner.py:85-106``)."""

from __future__ import annotations

import platform


def provenance(dev=None) -> dict:
    import torch

    out = {"torch": torch.__version__, "cuda_runtime": torch.version.cuda, "python": platform.python_version(),
           "host": platform.node()}
    try:
        out["nccl"] = ".".join(str(x) for x in torch.cuda.nccl.version())
    except Exception:   # noqa: BLE001  (CPU-only builds)
        pass
    if torch.cuda.is_available():
        d = torch.device("cuda", torch.cuda.current_device()) if dev is None else torch.device(dev)
        p = torch.cuda.get_device_properties(d)
        out.update(gpu=p.name, sm=f"{p.major}.{p.minor}", sms=p.multi_processor_count,
                   hbm_gib=round(p.total_memory / 2 ** 30, 1), gpus_visible=torch.cuda.device_count())
        try:
            import pynvml

            pynvml.nvmlInit()
            out["driver"] = pynvml.nvmlSystemGetDriverVersion()
            pynvml.nvmlShutdown()
        except Exception:   # noqa: BLE001  (no NVML: leave the driver out)
            pass
    return out
