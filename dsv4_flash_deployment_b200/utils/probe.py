"""Hardware probe of a B200 node: the facts this engine's kernels and layouts
depend on, one isolated check each, written as JSON.

Checks (every one records ``ok``, its seconds and its result or error, so one
failure does not hide the others):

  software     torch / CUDA runtime / NCCL / Python versions, this library's extension
  devices      per GPU: name, compute capability (sm_100 expected), SMs, HBM, L2
  nvml         per GPU, read only: SM / memory clocks and their maxima, power draw and
               limit, active clock-event reasons, temperature, ECC / persistence / MIG
               modes, NVLink links up
  peer_access  the peer-access matrix (every pair must be reachable for the NVLink paths)
  kernels      a small block-scaled FP8 GEMM of this library (tcgen05) against torch
  hbm          device-to-device copy bandwidth (``--hbm-gib`` per direction, CUDA events)
  peer_copy    copy bandwidth from GPU 0 to every other GPU (plain peer copies)
  storage      read throughput of ``--storage-path`` into pinned memory with the native
               reader, then host-to-device bandwidth of the same bytes

It changes no setting of any GPU (NVML is used only to read).  The reference
probes its TPU slices the same way before serving (``tpu-v7x/scripts/
probe_v7x.py``: device model and ordering, HBM, kernel lowering, remote DMA
bandwidth, HBM bandwidth, storage-to-HBM throughput, one JSON per process).

    python -m dsv4_flash_deployment_b200.utils.probe --out probe/ [--storage-path /ckpt/shard.safetensors]
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import socket
import time
import traceback


def _run(results: dict, name: str, fn, *args) -> None:
    t0 = time.perf_counter()
    try:
        results[name] = {"ok": True, **fn(*args)}
    except Exception as e:  # noqa: BLE001  (a probe records every failure and goes on)
        results[name] = {"ok": False, "error": f"{type(e).__name__}: {e}", "trace": traceback.format_exc()[-3000:]}
    results[name]["seconds"] = round(time.perf_counter() - t0, 3)
    print(f"[probe] {name}: ok={results[name]['ok']} ({results[name]['seconds']} s)", flush=True)


def _need_cuda():
    import torch

    if not torch.cuda.is_available():
        raise RuntimeError("no CUDA device")
    return torch


def check_software() -> dict:
    import torch

    out = {"torch": torch.__version__, "cuda_runtime": torch.version.cuda, "python": platform.python_version()}
    try:
        out["nccl"] = ".".join(str(x) for x in torch.cuda.nccl.version())
    except Exception as e:  # noqa: BLE001
        out["nccl"] = f"unavailable: {e}"
    from ..ops import _ext

    so = _ext.BUILD / f"{_ext.NAME}.so"
    out["extension"] = str(so) if so.exists() else "not built"
    return out


def check_devices() -> dict:
    torch = _need_cuda()
    devs = []
    for i in range(torch.cuda.device_count()):
        p = torch.cuda.get_device_properties(i)
        devs.append({"index": i, "name": p.name, "sm": f"{p.major}.{p.minor}", "sms": p.multi_processor_count,
                     "hbm_gib": round(p.total_memory / 2 ** 30, 1),
                     "l2_mib": round(getattr(p, "L2_cache_size", 0) / 2 ** 20, 1)})
    return {"count": len(devs), "devices": devs, "all_sm100": all(d["sm"] == "10.0" for d in devs)}


# clock-event reason bits (NVML's documented masks)
REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
           0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
           0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


def check_nvml(nvml=None) -> dict:
    """Read-only NVML queries per GPU (``nvml``: the pynvml module, or a stand-in)."""
    if nvml is None:
        import pynvml as nvml
    nvml.nvmlInit()
    try:
        gpus = []
        for i in range(nvml.nvmlDeviceGetCount()):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            g = {"index": i, "name": _s(nvml.nvmlDeviceGetName(h))}

            def q(key, fn, *a):
                try:
                    g[key] = fn(h, *a)
                except Exception as e:  # noqa: BLE001  (a query the driver does not support)
                    g[key] = f"n/a ({type(e).__name__})"
            q("sm_mhz", nvml.nvmlDeviceGetClockInfo, nvml.NVML_CLOCK_SM)
            q("sm_max_mhz", nvml.nvmlDeviceGetMaxClockInfo, nvml.NVML_CLOCK_SM)
            q("mem_mhz", nvml.nvmlDeviceGetClockInfo, nvml.NVML_CLOCK_MEM)
            q("power_mw", nvml.nvmlDeviceGetPowerUsage)
            q("power_limit_mw", nvml.nvmlDeviceGetPowerManagementLimit)
            q("temperature_c", nvml.nvmlDeviceGetTemperature, nvml.NVML_TEMPERATURE_GPU)
            q("persistence_mode", nvml.nvmlDeviceGetPersistenceMode)
            q("ecc_mode", lambda hh: list(nvml.nvmlDeviceGetEccMode(hh)))
            q("mig_mode", lambda hh: list(nvml.nvmlDeviceGetMigMode(hh)))
            try:
                bits = nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                g["clock_event_reasons"] = [n for b, n in REASONS.items() if bits & b]
            except Exception as e:  # noqa: BLE001
                g["clock_event_reasons"] = f"n/a ({type(e).__name__})"
            links = 0
            for link in range(getattr(nvml, "NVML_NVLINK_MAX_LINKS", 18)):
                try:
                    links += int(nvml.nvmlDeviceGetNvLinkState(h, link) == nvml.NVML_FEATURE_ENABLED)
                except Exception:  # noqa: BLE001  (past the last link)
                    break
            g["nvlink_links_up"] = links
            gpus.append(g)
        flags = sorted({r for g in gpus if isinstance(g.get("clock_event_reasons"), list)
                        for r in g["clock_event_reasons"]} & {"hw_slowdown", "hw_thermal_slowdown",
                                                               "sw_thermal_slowdown"})
        return {"driver": _s(nvml.nvmlSystemGetDriverVersion()), "gpus": gpus, "slowdown_reasons": flags}
    finally:
        nvml.nvmlShutdown()


def _s(x) -> str:
    return x.decode() if isinstance(x, bytes) else str(x)


def check_peer_access() -> dict:
    torch = _need_cuda()
    n = torch.cuda.device_count()
    m = [[i == j or bool(torch.cuda.can_device_access_peer(i, j)) for j in range(n)] for i in range(n)]
    return {"matrix": m, "all_pairs": all(all(r) for r in m)}


def check_kernels() -> dict:
    """One block-scaled FP8 GEMM of this library (TMA + tcgen05 + TMEM) against the
    fp32 oracle of the same op."""
    torch = _need_cuda()
    from ..ops import _ext
    from ..ops import gemm as G
    from ..ref import numerics as N

    _ext.load(required=True)
    g = torch.Generator().manual_seed(0)
    m, n, k = 256, 16, 512
    w = (torch.randn(m, k, generator=g) * 0.5).to(torch.float8_e4m3fn)
    s = torch.randint(118, 123, (m // 32, k // 32), generator=g, dtype=torch.int32).to(torch.uint8)
    x = torch.randn(n, k, generator=g).to(torch.bfloat16)
    want = N.fp8_linear(x, w, s, torch.float32)
    mw = G.MxWeight.from_checkpoint(w, s, "cuda:0")
    xq, xsf = G.quantize(x.to("cuda:0"))
    out = torch.empty(n, m, dtype=torch.float32, device="cuda:0")
    G.gemm_mx(xq, xsf, n, mw, out, G.EPI_F32)
    torch.cuda.synchronize()
    G.ErrorWord.check("cuda:0")
    got = out.cpu()
    rel = float((got - want).norm() / want.norm().clamp_min(1e-12))
    return {"gemm_mx8": {"m": m, "n": n, "k": k, "relative_error_vs_fp32": round(rel, 6)}, "ok_numerics": rel < 5e-3}


def _event_time(torch, fn, iters: int) -> float:
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fn()
    torch.cuda.synchronize()
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / 1e3 / iters


def check_hbm(gib: float) -> dict:
    torch = _need_cuda()
    n = int(gib * 2 ** 30) // 4
    a = torch.empty(n, dtype=torch.float32, device="cuda:0")
    b = torch.empty_like(a)
    dt = _event_time(torch, lambda: b.copy_(a), 5)
    del a, b
    return {"bytes_per_copy": n * 4, "copy_gbs": round(2 * n * 4 / dt / 1e9, 1), "note": "read + write bytes"}


def check_peer_copy(mib: int) -> dict:
    torch = _need_cuda()
    out = {}
    n = mib * 2 ** 20
    src = torch.empty(n, dtype=torch.uint8, device="cuda:0")
    for j in range(1, torch.cuda.device_count()):
        dst = torch.empty(n, dtype=torch.uint8, device=f"cuda:{j}")
        dt = _event_time(torch, lambda: dst.copy_(src), 5)
        out[f"0->{j}"] = round(n / dt / 1e9, 1)
        del dst
    return {"bytes": n, "gbs": out}


def check_storage(path: str | None) -> dict:
    if not path:
        return {"skipped": "no --storage-path"}
    import torch

    import ctypes

    from ..ops.host import lib

    size = os.path.getsize(path)
    buf = torch.empty(size, dtype=torch.uint8, pin_memory=torch.cuda.is_available())
    L = lib()
    offs = (ctypes.c_int64 * 1)(0)
    lens = (ctypes.c_int64 * 1)(size)
    dsts = (ctypes.c_void_p * 1)(buf.data_ptr())
    t0 = time.perf_counter()
    rc = L.dsv4_pread_many(path.encode(), 1, offs, lens, dsts, 16)
    read_s = time.perf_counter() - t0
    if rc != 0:
        raise OSError(f"native read failed ({rc})")
    out = {"bytes": size, "read_gbs": round(size / read_s / 1e9, 2)}
    if torch.cuda.is_available():
        d = torch.empty(size, dtype=torch.uint8, device="cuda:0")
        dt = _event_time(torch, lambda: d.copy_(buf, non_blocking=True), 3)
        out["h2d_gbs"] = round(size / dt / 1e9, 1)
    return out


def probe(a) -> dict:
    res: dict = {"host": socket.gethostname(), "time": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
                 "pid": os.getpid()}
    _run(res, "software", check_software)
    _run(res, "devices", check_devices)
    _run(res, "nvml", check_nvml)
    _run(res, "peer_access", check_peer_access)
    if not a.skip_kernels:
        _run(res, "kernels", check_kernels)
    _run(res, "hbm", check_hbm, a.hbm_gib)
    _run(res, "peer_copy", check_peer_copy, a.peer_mib)
    _run(res, "storage", check_storage, a.storage_path)
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--out", default=None, help="directory of probe_<host>_<pid>.json (default: print only)")
    ap.add_argument("--hbm-gib", type=float, default=2.0)
    ap.add_argument("--peer-mib", type=int, default=256)
    ap.add_argument("--storage-path", default=None)
    ap.add_argument("--skip-kernels", action="store_true")
    a = ap.parse_args(argv)
    res = probe(a)
    text = json.dumps(res, indent=1, default=str)
    if a.out:
        os.makedirs(a.out, exist_ok=True)
        with open(os.path.join(a.out, f"probe_{res['host']}_{res['pid']}.json"), "w") as f:
            f.write(text + "\n")
    print(json.dumps({k: v.get("ok") for k, v in res.items() if isinstance(v, dict)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
