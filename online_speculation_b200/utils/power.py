"""GPU power / utilisation monitor for training runs (reads nvidia-smi; changes no GPU setting).

One ``nvidia-smi --query-gpu=... -lms <interval>`` process streams CSV samples for the chosen
device into a reader thread for the length of the run, so sampling costs one process instead
of one per sample.  :meth:`PowerMonitor.stop` ends the stream and summarises it: the energy
(trapezoid integral of the power samples over their timestamps), mean and peak power, mean
utilisation, peak memory and peak temperature.  A monitor that cannot start or parse reports
the error in its summary and never raises into the training loop.

Summary keys follow the reference GRPO script's power monitor
(experiments/arllm/train_gsm8k_grpo.py:67-159) so run manifests compare directly.
"""

from __future__ import annotations

import subprocess
import threading
import time
from typing import Any

QUERY = "power.draw,utilization.gpu,memory.used,temperature.gpu"


class PowerMonitor:
    def __init__(self, device_index: int = 0, interval_seconds: float = 1.0, *, command: list[str] | None = None):
        if interval_seconds <= 0:
            raise ValueError("the sampling interval has to be positive")
        self.interval_seconds = float(interval_seconds)
        self.command = command or ["nvidia-smi", f"--id={int(device_index)}", f"--query-gpu={QUERY}",
                                   "--format=csv,noheader,nounits", f"-lms={max(1, int(interval_seconds * 1000))}"]
        self.samples: list[tuple[float, float, float, float, float]] = []   # (t, W, util %, MiB, C)
        self.error: str | None = None
        self._proc: subprocess.Popen | None = None
        self._thread: threading.Thread | None = None
        self._t0 = 0.0

    def _read(self) -> None:
        assert self._proc is not None and self._proc.stdout is not None
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            try:
                w, u, m, c = (float(p) for p in parts[:4])
            except ValueError:
                if line.strip():
                    self.error = f"unparsed sample: {line.strip()[:80]}"
                continue
            self.samples.append((time.perf_counter() - self._t0, w, u, m, c))

    def start(self) -> "PowerMonitor":
        self._t0 = time.perf_counter()
        try:
            self._proc = subprocess.Popen(self.command, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
                                          bufsize=1)
        except OSError as err:                         # no nvidia-smi: the run goes on unmonitored
            self.error = f"{type(err).__name__}: {err}"
            return self
        self._thread = threading.Thread(target=self._read, name="power-monitor", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> dict[str, Any]:
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                self._proc.wait(timeout=5)
        if self._thread is not None:
            self._thread.join(timeout=5)
        s = list(self.samples)
        energy_wh = sum((b[0] - a[0]) / 3600.0 * (a[1] + b[1]) / 2.0 for a, b in zip(s, s[1:]))

        def agg(fn, k):
            return fn(x[k] for x in s) if s else None

        return {"sample_interval_seconds": self.interval_seconds, "samples": len(s),
                "gpu_power_integral_wh": energy_wh,
                "mean_power_watts": (sum(x[1] for x in s) / len(s)) if s else None,
                "peak_power_watts": agg(max, 1),
                "mean_utilization_percent": (sum(x[2] for x in s) / len(s)) if s else None,
                "peak_nvidia_smi_memory_mib": agg(max, 3), "peak_temperature_c": agg(max, 4),
                "monitor_error": self.error}

    def __enter__(self) -> "PowerMonitor":
        return self.start()

    def __exit__(self, *exc) -> None:
        self.stop()
