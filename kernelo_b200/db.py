"""SQLite results store.

Every measurement row points at its problem, its config and its run, and the
run carries the GPU, driver, CUDA, torch and native-library versions. The
schema text is the reference's (``kernelforge/db.py:35-99``: runs / problems /
configs / results, configs stored as a JSON parameter set plus a content
digest), so databases of the two implementations answer the same queries.
The ``triton_version`` column of ``runs`` records the native library version
here. The access layer is this project's own: interned problem and config
rows, one transaction per write, and the best-per-label ranking done in SQL
with a window function.
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

    def columns(self) -> dict[str, Any]:
        """The ``results`` columns this measurement fills (ids excluded).

        Times are stored in microseconds; a measurement that never ran has
        NULL timing and correctness columns."""
        t, v = self.timing, self.verification
        cols: dict[str, Any] = {"label": self.label, "status": self.status,
                                "correct": None if v is None else int(v.passed),
                                "rel_error": None if v is None else v.error,
                                "tflops": self.tflops, "gbps": self.gbps, "error": self.error}
        for stat in _TIMING_STATS:
            cols[f"{stat}_us"] = None if t is None else 1e3 * getattr(t, f"{stat}_ms")
        for name in ("warmup", "iterations", "timer"):
            cols[name] = None if t is None else getattr(t, name)
        cols["flushed_l2"] = None if t is None else int(t.flushed_l2)
        return cols


_TIMING_STATS = ("median", "mean", "std", "min", "max", "p95", "p99")
_RUN_ENV_COLUMNS = ("timestamp", "hostname", "platform", "python_version", "torch_version", "triton_version",
                    "cuda_version", "driver_version", "gpu_name", "gpu_arch", "gpu_memory_bytes", "sm_count",
                    "device_key")


def default_db_path() -> Path:
    configured = os.environ.get("KERNELFORGE_DB")
    return Path(configured) if configured else DEFAULT_DB_PATH


class ResultsDB:
    """The results store: one SQLite file in the reference's schema.

    Problems and configs are interned (one row each, looked up by their
    natural key and memoised per connection); every write is one transaction.
    """

    def __init__(self, path: str | Path | None = None) -> None:
        self.path = Path(path) if path is not None else default_db_path()
        if str(self.path) != ":memory:":
            self.path.parent.mkdir(parents=True, exist_ok=True)
        self._conn = sqlite3.connect(str(self.path))
        self._conn.row_factory = sqlite3.Row
        self._ids: dict[tuple, int] = {}
        try:
            self._prepare()
        except BaseException:
            self._conn.close()
            raise

    def _prepare(self) -> None:
        conn = self._conn
        conn.execute("PRAGMA foreign_keys = ON")
        found = conn.execute("PRAGMA user_version").fetchone()[0]
        if found not in (0, SCHEMA_VERSION):
            raise RuntimeError(f"{self.path} was written by schema version {found}, "
                               f"this build expects {SCHEMA_VERSION}")
        with conn:
            conn.executescript(_SCHEMA)
            conn.execute(f"PRAGMA user_version = {SCHEMA_VERSION}")

    def __enter__(self) -> ResultsDB:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()

    def close(self) -> None:
        self._conn.close()

    # ------------------------------------------------------------ writes
    def _insert(self, table: str, values: dict[str, Any]) -> int:
        names = ", ".join(values)
        marks = ", ".join("?" for _ in values)
        cursor = self._conn.execute(f"INSERT INTO {table} ({names}) VALUES ({marks})", tuple(values.values()))
        return int(cursor.lastrowid)

    def _intern(self, table: str, id_column: str, key: dict[str, Any], extra: dict[str, Any]) -> int:
        """The id of the row of ``table`` with natural key ``key``, inserted if new."""
        memo = (table, *key.values())
        if memo in self._ids:
            return self._ids[memo]
        where = " AND ".join(f"{name} = ?" for name in key)
        row = self._conn.execute(f"SELECT {id_column} FROM {table} WHERE {where}", tuple(key.values())).fetchone()
        rowid = int(row[0]) if row is not None else self._insert(table, {**key, **extra})
        self._ids[memo] = rowid
        return rowid

    def start_run(self, env: Environment, *, notes: str = "", version: str = "") -> int:
        with self._conn:
            return self._insert("runs", {**{name: getattr(env, name) for name in _RUN_ENV_COLUMNS},
                                         "kernelforge_version": version, "notes": notes})

    def problem_id(self, problem: Problem) -> int:
        return self._intern("problems", "problem_id",
                            {"operation": problem.operation, "shape_key": problem.shape_key,
                             "dtype": problem.dtype_name},
                            {"dims_json": json.dumps(problem.dims_dict, sort_keys=True)})

    def config_id(self, config: KernelConfig) -> int:
        return self._intern("configs", "config_id", {"operation": config.operation, "digest": config.digest},
                            {"params_json": config.to_json()})

    def _record(self, run_id: int, problem: Problem, m: Measurement) -> int:
        ids = {"run_id": run_id, "problem_id": self.problem_id(problem),
               "config_id": None if m.config is None else self.config_id(m.config)}
        return self._insert("results", {**ids, **m.columns()})

    def record(self, run_id: int, problem: Problem, m: Measurement) -> int:
        with self._conn:
            return self._record(run_id, problem, m)

    def record_many(self, run_id: int, problem: Problem, measurements: Iterable[Measurement]) -> None:
        with self._conn:
            for m in measurements:
                self._record(run_id, problem, m)

    # ------------------------------------------------------------ reads
    def _select(self, filters: dict[str, Any], *, tail: str = "ORDER BY r.result_id") -> list[dict]:
        where = " AND ".join(f"{column} = ?" for column in filters)
        query = f"{_JOINED} {'WHERE ' + where if where else ''} {tail}"
        return [dict(row) for row in self._conn.execute(query, tuple(filters.values()))]

    def _lookup_filters(self, problem: Problem, config: KernelConfig, label: str) -> dict[str, Any]:
        return {"p.operation": problem.operation, "p.shape_key": problem.shape_key, "p.dtype": problem.dtype_name,
                "c.digest": config.digest, "r.label": label}

    def has_result(self, problem: Problem, config: KernelConfig, *, label: str = "kernelforge") -> bool:
        """Whether (problem, config) already has a row: lets a sweep resume."""
        return bool(self._select(self._lookup_filters(problem, config, label), tail="LIMIT 1"))

    def latest_result(self, problem: Problem, config: KernelConfig, *, device_key: str,
                      label: str = "kernelforge") -> dict | None:
        """The newest row for (problem, config, label) measured on ``device_key``,
        or None: what a resumed sweep reuses instead of measuring again."""
        found = self._select({**self._lookup_filters(problem, config, label), "run.device_key": device_key},
                             tail="ORDER BY r.result_id DESC LIMIT 1")
        return found[0] if found else None

    def rows(self, *, operation: str | None = None, dtype: str | None = None) -> list[dict]:
        filters = {column: value for column, value in (("p.operation", operation), ("p.dtype", dtype)) if value}
        return self._select(filters)

    def best_per_label(self, *, operation: str | None = None) -> list[dict]:
        """Fastest correct row per (operation, shape, dtype, label), ranked in SQL."""
        where = "WHERE r.median_us IS NOT NULL AND (r.correct IS NULL OR r.correct != 0)"
        args: tuple = ()
        if operation:
            where += " AND p.operation = ?"
            args = (operation,)
        query = (f"SELECT * FROM (SELECT j.*, ROW_NUMBER() OVER (PARTITION BY operation, shape_key, dtype, label "
                 f"ORDER BY median_us, result_id) AS rank_in_label FROM ({_JOINED} {where}) AS j) "
                 "WHERE rank_in_label = 1 ORDER BY operation, dtype, shape_key, label")
        found = []
        for row in self._conn.execute(query, args):
            item = dict(row)
            item.pop("rank_in_label")
            found.append(item)
        return found

    def runs(self) -> list[dict]:
        return [dict(row) for row in self._conn.execute("SELECT * FROM runs ORDER BY run_id")]

    def counts(self) -> dict[str, int]:
        tables = ("runs", "problems", "configs", "results")
        query = " UNION ALL ".join(f"SELECT '{t}', COUNT(*) FROM {t}" for t in tables)
        return {name: int(n) for name, n in self._conn.execute(query)}

    def operations(self) -> list[str]:
        return [row[0] for row in self._conn.execute("SELECT DISTINCT operation FROM problems ORDER BY operation")]
