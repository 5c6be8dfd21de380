"""Hardware counters for one launch, through Nsight Compute.

The reference profiles a kernel by re-running its CLI under ``ncu`` with named
sections and parsing the raw CSV page (``kernelforge/profiling/nsight.py``);
this module keeps that interface -- the section names a user passes
(``throughput``, ``memory``, ...), :func:`build_command`, :func:`run` and
:class:`NsightRun` -- and builds it around a :class:`Capture` description that
knows the rules this pool imposes on a capture:

* every command carries ``--clock-control none``: without it ncu locks the
  GPU's clocks for the capture, and an interrupted capture can leave them
  locked for the GPU's next user;
* the target runs once without ncu first and is only profiled if that run
  exited 0, so a program that faults is never replayed under the profiler;
* a capture is one launch by default, and no timeout is put on ncu (killing it
  mid-capture can leave the GPU unusable): keep the profiled case small.
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

#: Non-metric columns of the raw page worth keeping beside the counters.
_KEPT_COLUMNS = frozenset({"Grid Size", "Block Size", "Registers Per Thread"})


def ncu_available() -> bool:
    return shutil.which("ncu") is not None


@dataclass(frozen=True)
class Capture:
    """One ncu invocation: what to run, which sections, which launches."""

    target: tuple[str, ...]
    sections: tuple[str, ...] = DEFAULT_SECTIONS
    kernel_filter: str | None = None
    launch_count: int = 1
    launch_skip: int = 0
    report_path: Path | None = None

    def __post_init__(self) -> None:
        unknown = sorted(set(self.sections).difference(SECTIONS))
        if unknown:
            raise ValueError(f"unknown sections {unknown}; available: {sorted(SECTIONS)}")
        if self.launch_count < 1:
            raise ValueError("launch_count must be at least 1")

    def argv(self) -> list[str]:
        opts = ["--clock-control", "none", "--target-processes", "all"]
        opts += [arg for name in self.sections for arg in ("--section", SECTIONS[name])]
        if self.kernel_filter:
            opts += ["--kernel-name", self.kernel_filter]
        opts += ["--launch-count", str(self.launch_count), "--launch-skip", str(self.launch_skip)]
        if self.report_path is not None:
            opts += ["--export", str(self.report_path), "--force-overwrite"]
        return ["ncu", *opts, "--csv", "--page", "raw", *self.target]


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
        out = io.StringIO()
        out.write("$ " + " ".join(self.command) + "\n")
        if not self.ok:
            out.write(f"exited {self.returncode}\n")
            out.write(self.stderr.strip()[-2000:])
            return out.getvalue().rstrip()
        if not self.metrics:
            out.write(self.stdout.strip() + "\n")
        for kernel, counters in self.metrics.items():
            out.write(f"\n{kernel}\n")
            pad = max(map(len, counters), default=0)
            for name in counters:
                out.write(f"  {name.ljust(pad)}  {counters[name]}\n")
        if self.report_path is not None:
            out.write(f"\nreport: {self.report_path}\n")
        return out.getvalue().rstrip()


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
    return Capture(tuple(target), tuple(sections), kernel_filter, launch_count, launch_skip,
                   Path(report_path) if report_path is not None else None).argv()


def self_command(argv: list[str]) -> list[str]:
    """The command that re-runs this package's CLI with ``argv``."""
    return [sys.executable, "-m", "kernelo_b200", *argv]


def parse_raw_csv(stdout: str) -> dict[str, dict[str, str]]:
    """``ncu --csv --page raw`` text as {kernel: {metric: "value unit"}}.

    The page is a header row of metric names, a row of units and one row per
    profiled launch (ncu's own log lines, which do not start with a quote,
    are skipped). A kernel seen twice gets ``#<launch>`` appended. Anything
    not in that form parses to {} and the caller keeps the raw text."""
    body = "\n".join(line for line in stdout.splitlines() if line.startswith('"'))
    try:
        table = list(csv.reader(io.StringIO(body)))
    except csv.Error:
        return {}
    if len(table) < 3 or "Kernel Name" not in table[0]:
        return {}
    header, units, launches = table[0], table[1], table[2:]
    keep = [i for i, name in enumerate(header) if "__" in name or name in _KEPT_COLUMNS]
    name_at = header.index("Kernel Name")
    parsed: dict[str, dict[str, str]] = {}
    for launch, row in enumerate(launches):
        if len(row) != len(header):
            continue
        kernel = row[name_at] if row[name_at] not in parsed else f"{row[name_at]} #{launch}"
        parsed[kernel] = {header[i]: f"{row[i]} {units[i]}".strip() for i in keep}
    return parsed


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
    capture = Capture(tuple(target), tuple(sections), kernel_filter, launch_count, launch_skip,
                      Path(report_path) if report_path is not None else None)
    plain = subprocess.run(list(target), capture_output=True, text=True)
    if plain.returncode != 0:
        return NsightRun(tuple(target), plain.returncode, plain.stdout,
                         "not profiled: the plain run failed\n" + plain.stderr)
    command = capture.argv()
    done = subprocess.run(command, capture_output=True, text=True)
    return NsightRun(tuple(command), done.returncode, done.stdout, done.stderr, capture.report_path,
                     parse_raw_csv(done.stdout) if done.returncode == 0 else {})
