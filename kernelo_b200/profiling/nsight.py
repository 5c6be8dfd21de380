"""Nsight Compute counters for one launch (``kernelforge/profiling/nsight.py``).

The latency harness says which configuration is faster; the counters say why
(tensor-pipe and DRAM throughput against peak, occupancy, warp stalls). Sections
are requested by name, as in the reference, and the raw page is parsed into
{kernel: {metric: value}}.

Two rules are built in rather than left to the caller:

* ``--clock-control none`` on every command. Without it ncu locks the GPU's
  clocks for the capture, and a capture that is interrupted can leave them
  locked for whoever uses the GPU next.
* The target runs once without ncu first, and is profiled only if that run
  exited 0: a program that faults must not be replayed under the profiler.

Keep captures small (one launch of one kernel, inputs of a few GB at most):
each captured launch is replayed once per hardware pass (a full set is ~40).
No timeout is imposed on the ncu process, since killing ncu in the middle of
a capture can leave the GPU unusable; a small capture ends by itself.
"""

from __future__ import annotations

import csv
import io
import shutil
import subprocess
import sys
from dataclasses import dataclass, field
from pathlib import Path

#: Nsight Compute sections, keyed by the question each answers.
SECTIONS: dict[str, str] = {
    "launch": "LaunchStats",
    "occupancy": "Occupancy",
    "memory": "MemoryWorkloadAnalysis",
    "throughput": "SpeedOfLight",
    "stalls": "WarpStateStats",
    "instructions": "InstructionStats",
}

DEFAULT_SECTIONS = ("launch", "occupancy", "throughput", "memory", "stalls")


def ncu_available() -> bool:
    return shutil.which("ncu") is not None


@dataclass(frozen=True)
class NsightRun:
    command: tuple[str, ...]
    returncode: int
    stdout: str
    stderr: str
    report_path: Path | None = None
    metrics: dict[str, dict[str, str]] = field(default_factory=dict)

    @property
    def ok(self) -> bool:
        return self.returncode == 0

    def render(self) -> str:
        lines = [f"$ {' '.join(self.command)}"]
        if not self.ok:
            lines.append(f"exited {self.returncode}")
            if self.stderr.strip():
                lines.append(self.stderr.strip()[-2000:])
            return "\n".join(lines)
        for kernel, values in self.metrics.items():
            lines.append(f"\n{kernel}")
            width = max((len(k) for k in values), default=0)
            lines.extend(f"  {k:<{width}}  {v}" for k, v in values.items())
        if not self.metrics:
            lines.append(self.stdout.strip())
        if self.report_path is not None:
            lines.append(f"\nreport: {self.report_path}")
        return "\n".join(lines)


def build_command(
    target: list[str],
    *,
    sections: tuple[str, ...] = DEFAULT_SECTIONS,
    kernel_filter: str | None = None,
    launch_count: int = 1,
    launch_skip: int = 0,
    report_path: str | Path | None = None,
) -> list[str]:
    """The ncu command line that profiles ``target`` (clocks never locked)."""
    unknown = sorted(set(sections) - set(SECTIONS))
    if unknown:
        raise ValueError(f"unknown sections {unknown}; available: {sorted(SECTIONS)}")
    if launch_count < 1:
        raise ValueError("launch_count must be at least 1")
    command = ["ncu", "--clock-control", "none", "--target-processes", "all"]
    for name in sections:
        command += ["--section", SECTIONS[name]]
    if kernel_filter:
        command += ["--kernel-name", kernel_filter]
    command += ["--launch-count", str(launch_count), "--launch-skip", str(launch_skip)]
    if report_path is not None:
        command += ["--export", str(report_path), "--force-overwrite"]
    command += ["--csv", "--page", "raw"]
    return command + list(target)


def self_command(argv: list[str]) -> list[str]:
    """The command that re-runs this package's CLI with ``argv``."""
    return [sys.executable, "-m", "kernelo_b200", *argv]


def parse_raw_csv(stdout: str) -> dict[str, dict[str, str]]:
    """``ncu --csv --page raw``: a header of metric names, a row of units, then
    one row per profiled launch. Returns {kernel: {metric: "value unit"}};
    empty if the text is not in that form (the caller keeps the raw text)."""
    lines = [ln for ln in stdout.splitlines() if ln.startswith('"')]
    try:
        rows = list(csv.reader(io.StringIO("\n".join(lines))))
    except csv.Error:
        return {}
    if len(rows) < 3:
        return {}
    header, units = rows[0], rows[1]
    try:
        name_col = header.index("Kernel Name")
    except ValueError:
        return {}
    out: dict[str, dict[str, str]] = {}
    for i, row in enumerate(rows[2:]):
        if len(row) != len(header):
            continue
        kernel = f"{row[name_col]} #{i}" if row[name_col] in out else row[name_col]
        out[kernel] = {
            h: f"{v} {u}".strip() for h, u, v in zip(header, units, row)
            if "__" in h or h in ("Grid Size", "Block Size", "Registers Per Thread")
        }
    return out


def run(
    target: list[str],
    *,
    sections: tuple[str, ...] = DEFAULT_SECTIONS,
    kernel_filter: str | None = None,
    launch_count: int = 1,
    launch_skip: int = 0,
    report_path: str | Path | None = None,
) -> NsightRun:
    """Run ``target`` once plainly, then, if it exited 0, under Nsight Compute."""
    if not ncu_available():
        raise RuntimeError("ncu was not found on PATH; install NVIDIA Nsight Compute to collect counters")
    plain = subprocess.run(list(target), capture_output=True, text=True)
    if plain.returncode != 0:
        return NsightRun(tuple(target), plain.returncode, plain.stdout,
                         "not profiled: the plain run failed\n" + plain.stderr)
    command = build_command(target, sections=sections, kernel_filter=kernel_filter,
                            launch_count=launch_count, launch_skip=launch_skip, report_path=report_path)
    result = subprocess.run(command, capture_output=True, text=True)
    return NsightRun(
        command=tuple(command),
        returncode=result.returncode,
        stdout=result.stdout,
        stderr=result.stderr,
        report_path=Path(report_path) if report_path else None,
        metrics=parse_raw_csv(result.stdout) if result.returncode == 0 else {},
    )
