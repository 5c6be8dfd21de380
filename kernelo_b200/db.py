"""SQLite results store (``kernelforge/db.py:1-320``).

Every measurement row points at its problem, its config and its run, and the
run carries the GPU, driver, CUDA, torch and native-library versions. The
schema is the reference's (runs / problems / configs / results, configs stored
as a JSON parameter set plus a content digest), so databases from the two
implementations can be compared with the same queries. The ``triton_version``
column of ``runs`` records the native library version here.
"""

from __future__ import annotations

import json
import os
import sqlite3
from collections.abc import Iterable
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from kernelo_b200.runtime.env import Environment
from kernelo_b200.testing import VerificationResult
from kernelo_b200.tuning.config import KernelConfig, Problem

SCHEMA_VERSION = 1
DEFAULT_DB_PATH = Path("results/kernelforge.db")

_SCHEMA = """
CREATE TABLE IF NOT EXISTS runs (
    run_id              INTEGER PRIMARY KEY AUTOINCREMENT,
    timestamp           TEXT    NOT NULL,
    hostname            TEXT,
    platform            TEXT,
    python_version      TEXT,
    torch_version       TEXT,
    triton_version      TEXT,
    cuda_version        TEXT,
    driver_version      TEXT,
    gpu_name            TEXT,
    gpu_arch            TEXT,
    gpu_memory_bytes    INTEGER,
    sm_count            INTEGER,
    device_key          TEXT    NOT NULL,
    kernelforge_version TEXT,
    notes               TEXT    NOT NULL DEFAULT ''
);
CREATE TABLE IF NOT EXISTS problems (
    problem_id INTEGER PRIMARY KEY AUTOINCREMENT,
    operation  TEXT NOT NULL,
    shape_key  TEXT NOT NULL,
    dtype      TEXT NOT NULL,
    dims_json  TEXT NOT NULL,
    UNIQUE (operation, shape_key, dtype)
);
CREATE TABLE IF NOT EXISTS configs (
    config_id   INTEGER PRIMARY KEY AUTOINCREMENT,
    operation   TEXT NOT NULL,
    digest      TEXT NOT NULL,
    params_json TEXT NOT NULL,
    UNIQUE (operation, digest)
);
CREATE TABLE IF NOT EXISTS results (
    result_id  INTEGER PRIMARY KEY AUTOINCREMENT,
    run_id     INTEGER NOT NULL REFERENCES runs (run_id),
    problem_id INTEGER NOT NULL REFERENCES problems (problem_id),
    config_id  INTEGER          REFERENCES configs (config_id),
    label      TEXT    NOT NULL,
    status     TEXT    NOT NULL,
    correct    INTEGER,
    rel_error  REAL,
    median_us  REAL,
    mean_us    REAL,
    std_us     REAL,
    min_us     REAL,
    max_us     REAL,
    p95_us     REAL,
    p99_us     REAL,
    warmup     INTEGER,
    iterations INTEGER,
    timer      TEXT,
    flushed_l2 INTEGER,
    tflops     REAL,
    gbps       REAL,
    error      TEXT NOT NULL DEFAULT ''
);
CREATE INDEX IF NOT EXISTS idx_results_problem ON results (problem_id, label);
CREATE INDEX IF NOT EXISTS idx_results_run     ON results (run_id);
"""

_JOINED = """
SELECT r.result_id, r.label, r.status, r.correct, r.rel_error,
       r.median_us, r.mean_us, r.std_us, r.min_us, r.max_us, r.p95_us, r.p99_us,
       r.warmup, r.iterations, r.timer, r.flushed_l2, r.tflops, r.gbps, r.error,
       p.operation, p.shape_key, p.dtype, p.dims_json,
       c.params_json, c.digest,
       run.run_id, run.timestamp, run.gpu_name, run.gpu_arch, run.device_key,
       run.torch_version, run.triton_version, run.cuda_version, run.driver_version
FROM results AS r
JOIN problems AS p   ON p.problem_id = r.problem_id
JOIN runs     AS run ON run.run_id   = r.run_id
LEFT JOIN configs AS c ON c.config_id = r.config_id
"""


@dataclass(frozen=True)
class Measurement:
    label: str
    status: str
    config: KernelConfig | None = None
    verification: VerificationResult | None = None
    timing: Any = None
    tflops: float | None = None
    gbps: float | None = None
    error: str = ""


def default_db_path() -> Path:
    return Path(os.environ.get("KERNELFORGE_DB", str(DEFAULT_DB_PATH)))


def _us(timing: Any, attr: str) -> float | None:
    return None if timing is None else getattr(timing, attr) * 1e3


class ResultsDB:
    def __init__(self, path: str | Path | None = None) -> None:
        self.path = Path(path) if path is not None else default_db_path()
        if str(self.path) != ":memory:":
            self.path.parent.mkdir(parents=True, exist_ok=True)
        self._conn = sqlite3.connect(str(self.path))
        self._conn.row_factory = sqlite3.Row
        self._conn.execute("PRAGMA foreign_keys = ON")
        self._conn.executescript(_SCHEMA)
        version = int(self._conn.execute("PRAGMA user_version").fetchone()[0])
        if version == 0:
            self._conn.execute(f"PRAGMA user_version = {SCHEMA_VERSION}")
        elif version != SCHEMA_VERSION:
            self._conn.close()
            raise RuntimeError(
                f"{self.path} was written by schema version {version}, "
                f"this build expects {SCHEMA_VERSION}"
            )
        self._conn.commit()

    def __enter__(self) -> ResultsDB:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()

    def close(self) -> None:
        self._conn.close()

    # writes -----------------------------------------------------------------
    def start_run(self, env: Environment, *, notes: str = "", version: str = "") -> int:
        cols = (
            "timestamp, hostname, platform, python_version, torch_version, triton_version, "
            "cuda_version, driver_version, gpu_name, gpu_arch, gpu_memory_bytes, sm_count, "
            "device_key, kernelforge_version, notes"
        )
        values = (
            env.timestamp, env.hostname, env.platform, env.python_version, env.torch_version,
            env.triton_version, env.cuda_version, env.driver_version, env.gpu_name, env.gpu_arch,
            env.gpu_memory_bytes, env.sm_count, env.device_key, version, notes,
        )
        cur = self._conn.execute(f"INSERT INTO runs ({cols}) VALUES ({','.join('?' * 15)})", values)
        self._conn.commit()
        return int(cur.lastrowid)

    def problem_id(self, problem: Problem) -> int:
        key = (problem.operation, problem.shape_key, problem.dtype_name)
        self._conn.execute(
            "INSERT OR IGNORE INTO problems (operation, shape_key, dtype, dims_json) VALUES (?,?,?,?)",
            (*key, json.dumps(problem.dims_dict, sort_keys=True)),
        )
        row = self._conn.execute(
            "SELECT problem_id FROM problems WHERE operation=? AND shape_key=? AND dtype=?", key
        ).fetchone()
        return int(row[0])

    def config_id(self, config: KernelConfig) -> int:
        self._conn.execute(
            "INSERT OR IGNORE INTO configs (operation, digest, params_json) VALUES (?,?,?)",
            (config.operation, config.digest, config.to_json()),
        )
        row = self._conn.execute(
            "SELECT config_id FROM configs WHERE operation=? AND digest=?",
            (config.operation, config.digest),
        ).fetchone()
        return int(row[0])

    def record(self, run_id: int, problem: Problem, m: Measurement) -> int:
        t, v = m.timing, m.verification
        values = (
            run_id,
            self.problem_id(problem),
            None if m.config is None else self.config_id(m.config),
            m.label,
            m.status,
            None if v is None else int(v.passed),
            None if v is None else v.error,
            _us(t, "median_ms"),
            _us(t, "mean_ms"),
            _us(t, "std_ms"),
            _us(t, "min_ms"),
            _us(t, "max_ms"),
            _us(t, "p95_ms"),
            _us(t, "p99_ms"),
            None if t is None else t.warmup,
            None if t is None else t.iterations,
            None if t is None else t.timer,
            None if t is None else int(t.flushed_l2),
            m.tflops,
            m.gbps,
            m.error,
        )
        cur = self._conn.execute(
            "INSERT INTO results (run_id, problem_id, config_id, label, status, correct, rel_error, "
            "median_us, mean_us, std_us, min_us, max_us, p95_us, p99_us, warmup, iterations, timer, "
            f"flushed_l2, tflops, gbps, error) VALUES ({','.join('?' * 21)})",
            values,
        )
        self._conn.commit()
        return int(cur.lastrowid)

    def record_many(self, run_id: int, problem: Problem, measurements: Iterable[Measurement]) -> None:
        for m in measurements:
            self.record(run_id, problem, m)

    def has_result(self, problem: Problem, config: KernelConfig, *, label: str = "kernelforge") -> bool:
        """Whether (problem, config) already has a row: lets a sweep resume."""
        row = self._conn.execute(
            "SELECT 1 FROM results r JOIN problems p ON p.problem_id = r.problem_id "
            "JOIN configs c ON c.config_id = r.config_id WHERE p.operation=? AND p.shape_key=? "
            "AND p.dtype=? AND c.digest=? AND r.label=? LIMIT 1",
            (problem.operation, problem.shape_key, problem.dtype_name, config.digest, label),
        ).fetchone()
        return row is not None

    def latest_result(self, problem: Problem, config: KernelConfig, *, device_key: str,
                      label: str = "kernelforge") -> dict | None:
        """The newest row for (problem, config, label) measured on ``device_key``,
        or None: what a resumed sweep reuses instead of measuring again."""
        row = self._conn.execute(
            _JOINED + " WHERE p.operation=? AND p.shape_key=? AND p.dtype=? AND c.digest=? AND r.label=? "
            "AND run.device_key=? ORDER BY r.result_id DESC LIMIT 1",
            (problem.operation, problem.shape_key, problem.dtype_name, config.digest, label, device_key),
        ).fetchone()
        return None if row is None else dict(row)

    # reads ------------------------------------------------------------------
    def rows(self, *, operation: str | None = None, dtype: str | None = None) -> list[dict]:
        where, params = [], []
        if operation:
            where.append("p.operation = ?")
            params.append(operation)
        if dtype:
            where.append("p.dtype = ?")
            params.append(dtype)
        query = _JOINED + (" WHERE " + " AND ".join(where) if where else "") + " ORDER BY r.result_id"
        return [dict(r) for r in self._conn.execute(query, params)]

    def best_per_label(self, *, operation: str | None = None) -> list[dict]:
        """Fastest correct row per (operation, shape, dtype, label)."""
        best: dict[tuple, dict] = {}
        for row in self.rows(operation=operation):
            if row["median_us"] is None or row["correct"] == 0:
                continue
            key = (row["operation"], row["shape_key"], row["dtype"], row["label"])
            if key not in best or row["median_us"] < best[key]["median_us"]:
                best[key] = row
        return sorted(best.values(), key=lambda r: (r["operation"], r["dtype"], r["shape_key"], r["label"]))

    def runs(self) -> list[dict]:
        return [dict(r) for r in self._conn.execute("SELECT * FROM runs ORDER BY run_id")]

    def counts(self) -> dict[str, int]:
        return {
            t: int(self._conn.execute(f"SELECT COUNT(*) FROM {t}").fetchone()[0])
            for t in ("runs", "problems", "configs", "results")
        }

    def operations(self) -> list[str]:
        return [r[0] for r in self._conn.execute("SELECT DISTINCT operation FROM problems ORDER BY 1")]
