"""Reports from the results database (``kernelforge/benchmark/report.py:1-364``).

Every number a reader sees comes from rows in SQLite, with the GPU, driver and
library versions of the run that measured it. ``generate`` writes
``summary.md`` (environment, methodology warnings, one table per operation:
best median latency per implementation and shape, this build's throughput and
its speedup over PyTorch eager) and one CSV per operation.

The reference also draws figures with matplotlib; matplotlib is not installed
in this build's environment, so the report is tables only and says so.
"""

from __future__ import annotations

import csv
from dataclasses import dataclass, field
from pathlib import Path

from kernelo_b200.db import ResultsDB

#: Order in which implementations appear in tables (the reference's labels).
LABEL_ORDER = ("torch_eager", "torch_compile", "triton_baseline", "triton_autotune", "cuda", "kernelforge")
LABEL_TITLES = {
    "torch_eager": "PyTorch eager",
    "torch_compile": "torch.compile",
    "triton_baseline": "Triton (untuned)",
    "triton_autotune": "Triton autotune",
    "cuda": "CUDA (handwritten)",
    "kernelforge": "KernelForge B200",
}
MEMORY_BOUND_OPERATIONS = frozenset({"rmsnorm", "softmax", "vector_add", "gemv"})


@dataclass
class ReportArtifacts:
    directory: Path
    summary: Path
    tables: list[Path] = field(default_factory=list)
    notes: list[str] = field(default_factory=list)

    def render(self) -> str:
        lines = [f"Report written to {self.directory}", f"  {self.summary.name}"]
        lines += [f"  {p.name}" for p in self.tables]
        lines += [f"  note: {note}" for note in self.notes]
        return "\n".join(lines)


def _ordered_labels(labels) -> list[str]:
    present = set(labels)
    return [x for x in LABEL_ORDER if x in present] + sorted(present - set(LABEL_ORDER))


def _environment_section(db: ResultsDB) -> list[str]:
    runs = db.runs()
    if not runs:
        return ["No runs recorded."]
    latest = runs[-1]
    fields = (("GPU", "gpu_name"), ("Compute capability", "gpu_arch"), ("CUDA", "cuda_version"),
              ("Driver", "driver_version"), ("PyTorch", "torch_version"),
              ("Native library", "triton_version"))
    return ["| Field | Value |", "| --- | --- |"] + [f"| {t} | {latest.get(k) or '-'} |" for t, k in fields]


def _methodology_warnings(rows: list[dict]) -> list[str]:
    """Settings that make rows of one database incomparable."""
    warnings = []
    flushed = {r["flushed_l2"] for r in rows}
    if len(flushed) > 1:
        n = sum(1 for r in rows if r["flushed_l2"] == 1)
        warnings.append(f"this database mixes {n} L2-flushed measurement(s) with {len(rows) - n} unflushed; "
                        "the unflushed rows report a bandwidth the kernel would not see on cold inputs")
    timers = {r["timer"] for r in rows}
    if len(timers) > 1:
        warnings.append(f"this database mixes timers ({', '.join(sorted(str(t) for t in timers))}); "
                        "only cuda_event rows are GPU measurements")
    return warnings


def _summary_table(best: list[dict], operation: str) -> list[str]:
    rows = [r for r in best if r["operation"] == operation]
    if not rows:
        return []
    labels = _ordered_labels(r["label"] for r in rows)
    memory_bound = operation in MEMORY_BOUND_OPERATIONS
    metric_title, metric = ("GB/s", "gbps") if memory_bound else ("TFLOP/s", "tflops")
    header = ["shape", "dtype", *(LABEL_TITLES.get(x, x) + " (us)" for x in labels),
              f"KernelForge B200 {metric_title}", "speedup vs eager"]
    lines = ["| " + " | ".join(header) + " |", "| " + " | ".join(["---"] * len(header)) + " |"]
    groups: dict[tuple[str, str], dict[str, dict]] = {}
    for r in rows:
        groups.setdefault((r["shape_key"], r["dtype"]), {})[r["label"]] = r
    for (shape, dtype), by_label in groups.items():
        line = [shape, dtype] + [f"{by_label[x]['median_us']:.1f}" if x in by_label else "-" for x in labels]
        mine = by_label.get("kernelforge")
        line.append(f"{mine[metric]:.1f}" if mine and mine.get(metric) else "-")
        eager = by_label.get("torch_eager")
        line.append(f"{eager['median_us'] / mine['median_us']:.2f}x" if mine and eager else "-")
        lines.append("| " + " | ".join(line) + " |")
    return lines


def _write_csv(path: Path, rows: list[dict]) -> None:
    columns = ["operation", "shape_key", "dtype", "label", "median_us", "p99_us", "tflops", "gbps", "rel_error",
               "timer", "flushed_l2", "params_json", "gpu_name", "timestamp"]
    with path.open("w", newline="") as fh:
        writer = csv.DictWriter(fh, fieldnames=columns, extrasaction="ignore")
        writer.writeheader()
        writer.writerows(rows)


def generate(db: ResultsDB, directory: str | Path = "reports", *,
             operations: list[str] | None = None) -> ReportArtifacts:
    """Write ``summary.md`` and one CSV per operation into ``directory``."""
    out = Path(directory)
    out.mkdir(parents=True, exist_ok=True)
    artifacts = ReportArtifacts(directory=out, summary=out / "summary.md")
    artifacts.notes.append("tables only: figures need matplotlib, which is not installed")
    rows = [r for r in db.rows() if r["median_us"] is not None and r["correct"] != 0]
    if not rows:
        artifacts.summary.write_text("# KernelForge B200 results\n\nNo correct, timed measurements in the "
                                     "database yet. Run `python -m kernelo_b200 tune` or `benchmark` first.\n")
        artifacts.notes.append("database contained no usable measurements")
        return artifacts
    best = db.best_per_label()
    present = operations or sorted({r["operation"] for r in rows})
    lines = ["# KernelForge B200 results", "",
             "Generated from the results database by `python -m kernelo_b200 report`. Latencies are "
             "medians over the iterations recorded with each row.", "",
             "## Environment", "", *_environment_section(db), ""]
    for warning in _methodology_warnings(rows):
        artifacts.notes.append(warning)
        lines += [f"> **Warning:** {warning}", ""]
    for operation in present:
        table = _summary_table(best, operation)
        if not table:
            continue
        lines += [f"## {operation}", "", *table, ""]
        export = out / f"{operation}.csv"
        _write_csv(export, [r for r in best if r["operation"] == operation])
        artifacts.tables.append(export)
    lines += ["## Files", "", *(f"- `{p.name}`" for p in artifacts.tables), ""]
    artifacts.summary.write_text("\n".join(lines))
    return artifacts
