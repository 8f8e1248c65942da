"""Metric logging fan-out (reference: ``Logger`` ``nemo_rl/utils/logger.py:1253``,
``LoggerInterface`` ``:136``, GPU monitor ``RayGpuMonitorLogger`` ``:792``).

Backends: stdout, JSONL (always available), TensorBoard (when the package is
importable).  W&B / MLflow / SwanLab keys in the config are accepted and
reported as unavailable when their packages are not installed.  Only rank 0
writes.  ``GpuMonitor`` samples utilisation / memory / clocks through NVML on a
background thread and logs them as ``gpu/*`` metrics.
"""

from __future__ import annotations

import json
import os
import threading
import time
from typing import Any, Optional

__all__ = ["Logger", "LoggerInterface", "JsonlLogger", "StdoutLogger", "TensorboardLogger", "GpuMonitor",
           "flatten_metrics"]


def _rank0() -> bool:
    try:
        import torch.distributed as dist

        return (not dist.is_initialized()) or dist.get_rank() == 0
    except Exception:  # noqa: BLE001
        return True


def flatten_metrics(d: dict, prefix: str = "") -> dict[str, float]:
    out = {}
    for k, v in d.items():
        key = f"{prefix}/{k}" if prefix else str(k)
        if isinstance(v, dict):
            out.update(flatten_metrics(v, key))
        elif isinstance(v, (int, float)) and not isinstance(v, bool):
            out[key] = float(v)
    return out


class LoggerInterface:
    def log_metrics(self, metrics: dict, step: int, prefix: str = "") -> None: ...

    def log_hyperparams(self, params: dict) -> None: ...

    def close(self) -> None: ...


class JsonlLogger(LoggerInterface):
    def __init__(self, log_dir: str):
        os.makedirs(log_dir, exist_ok=True)
        self.path = os.path.join(log_dir, "metrics.jsonl")
        self.f = open(self.path, "a")

    def log_metrics(self, metrics, step, prefix=""):
        self.f.write(json.dumps({"step": step, "time": time.time(), **flatten_metrics(metrics, prefix)}) + "\n")
        self.f.flush()

    def log_hyperparams(self, params):
        with open(os.path.join(os.path.dirname(self.path), "hparams.json"), "w") as f:
            json.dump(params, f, default=str, indent=1)

    def close(self):
        self.f.close()


class StdoutLogger(LoggerInterface):
    def __init__(self, keys: Optional[list[str]] = None):
        self.keys = keys

    def log_metrics(self, metrics, step, prefix=""):
        flat = flatten_metrics(metrics, prefix)
        if self.keys:
            flat = {k: v for k, v in flat.items() if any(k.endswith(s) for s in self.keys)}
        print(f"[step {step}] " + " ".join(f"{k}={v:.5g}" for k, v in sorted(flat.items())), flush=True)


class TensorboardLogger(LoggerInterface):
    def __init__(self, log_dir: str):
        from torch.utils.tensorboard import SummaryWriter

        self.w = SummaryWriter(log_dir=log_dir)

    def log_metrics(self, metrics, step, prefix=""):
        for k, v in flatten_metrics(metrics, prefix).items():
            self.w.add_scalar(k, v, step)
        self.w.flush()

    def log_hyperparams(self, params):
        self.w.add_text("hparams", json.dumps(params, default=str))

    def close(self):
        self.w.close()


class GpuMonitor:
    """Background NVML sampler; ``snapshot()`` returns the latest means."""

    def __init__(self, interval_s: float = 5.0):
        self.interval = interval_s
        self.samples: list[dict] = []
        self._stop = threading.Event()
        self._t: Optional[threading.Thread] = None

    def start(self) -> bool:
        try:
            import pynvml

            pynvml.nvmlInit()
        except Exception:  # noqa: BLE001 - no NVML: monitoring disabled
            return False
        self._nvml = pynvml
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return True

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            rec = {}
            for i in range(n.nvmlDeviceGetCount()):
                h = n.nvmlDeviceGetHandleByIndex(i)
                u = n.nvmlDeviceGetUtilizationRates(h)
                m = n.nvmlDeviceGetMemoryInfo(h)
                rec[f"gpu{i}/util"] = float(u.gpu)
                rec[f"gpu{i}/mem_used_gb"] = m.used / 1e9
                rec[f"gpu{i}/sm_mhz"] = float(n.nvmlDeviceGetClockInfo(h, n.NVML_CLOCK_SM))
            self.samples.append(rec)
            self._stop.wait(self.interval)

    def snapshot(self) -> dict:
        if not self.samples:
            return {}
        keys = self.samples[-1].keys()
        return {k: sum(s.get(k, 0.0) for s in self.samples) / len(self.samples) for k in keys}

    def stop(self):
        self._stop.set()


class Logger(LoggerInterface):
    """Fan-out logger configured like the reference's ``logger`` block."""

    def __init__(self, cfg: Optional[dict] = None):
        cfg = cfg or {}
        self.cfg = cfg
        self.backends: list[LoggerInterface] = []
        self.unavailable: list[str] = []
        log_dir = cfg.get("log_dir", "logs")
        if not _rank0():
            return
        self.backends.append(JsonlLogger(log_dir))
        if cfg.get("stdout", True):
            self.backends.append(StdoutLogger(cfg.get("stdout_keys")))
        if cfg.get("tensorboard_enabled", False):
            try:
                self.backends.append(TensorboardLogger(os.path.join(log_dir, "tensorboard")))
            except Exception as e:  # noqa: BLE001
                self.unavailable.append(f"tensorboard: {e}")
        for key, pkg in (("wandb_enabled", "wandb"), ("mlflow_enabled", "mlflow"), ("swanlab_enabled", "swanlab")):
            if cfg.get(key, False):
                self.unavailable.append(f"{pkg}: package not installed in this image")
        self.monitor = None
        if cfg.get("monitor_gpus", False):
            self.monitor = GpuMonitor(float(cfg.get("gpu_monitoring", {}).get("collection_interval", 5.0)))
            self.monitor.start()

    def log_metrics(self, metrics: dict, step: int, prefix: str = "") -> None:
        for b in self.backends:
            b.log_metrics(metrics, step, prefix)
        if getattr(self, "monitor", None) is not None and prefix == "train":
            snap = self.monitor.snapshot()
            if snap:
                for b in self.backends:
                    b.log_metrics(snap, step, "gpu")

    def log_hyperparams(self, params: dict) -> None:
        for b in self.backends:
            b.log_hyperparams(params)

    def close(self) -> None:
        for b in self.backends:
            b.close()
        if getattr(self, "monitor", None) is not None:
            self.monitor.stop()
