"""Command line interface, run as ``python -m kernelo_b200 <command>``.

The subcommands and flags are the reference's (``kernelforge/cli/main.py:542-631``:
``env``, ``tune`` with ``--explain``, ``benchmark``, ``compare``, ``profile``,
``report``, ``cache``), so scripts written against it keep working; each is a
thin layer over a library call that has tests of its own.

Structure: every subcommand is a :class:`Command` that declares its arguments
and runs against a :class:`Session` -- the parsed arguments plus the results
database and config cache, opened on first use and closed when the command
ends. Output goes through :class:`Table`, which sizes its columns to their
contents.
"""

from __future__ import annotations

import argparse
import sys
from collections.abc import Callable, Sequence
from pathlib import Path

from kernelo_b200 import __version__
from kernelo_b200.dtypes import SUPPORTED_DTYPES, parse_dtype
from kernelo_b200.tuning.config import Problem

#: Dimensions each operation takes, with the values used when a flag is absent.
_SHAPES: dict[str, dict[str, tuple[str, int]]] = {
    **{op: {"M": ("m", 2048), "N": ("n", 4096), "K": ("k", 4096)} for op in ("matmul", "fused_linear",
                                                                          "fused_linear_erf")},
    "gemv": {"M": ("m", 1), "N": ("n", 11008), "K": ("k", 4096)},
    **{op: {"rows": ("rows", 4096), "cols": ("cols", 4096)} for op in ("rmsnorm", "softmax")},
}

OPERATIONS = tuple(_SHAPES)


def build_problem(operation: str, args: argparse.Namespace) -> Problem:
    """The problem a command line describes: shape flags over the defaults."""
    try:
        dims = _SHAPES[operation]
    except KeyError:
        raise ValueError(f"unknown operation {operation!r}") from None
    sizes = {dim: getattr(args, flag, None) or default for dim, (flag, default) in dims.items()}
    return Problem.create(operation, parse_dtype(args.dtype), **sizes)


def heading(title: str) -> str:
    return f"\n{title}\n" + "-" * len(title)


class Table:
    """Rows printed under a header, each column as wide as its widest cell;
    numeric columns are right-aligned."""

    def __init__(self, *columns: str, right: Sequence[str] = ()) -> None:
        self.columns = columns
        self.right = set(right)
        self.rows: list[tuple[str, ...]] = []

    def add(self, *cells: object) -> None:
        self.rows.append(tuple(str(c) for c in cells))

    def render(self) -> str:
        widths = [max(len(col), *(len(r[i]) for r in self.rows)) if self.rows else len(col)
                  for i, col in enumerate(self.columns)]

        def line(cells):
            return "  ".join(c.rjust(w) if name in self.right else c.ljust(w)
                             for c, w, name in zip(cells, widths, self.columns)).rstrip()

        head = line(self.columns)
        return "\n".join([head, "-" * len(head), *(line(r) for r in self.rows)])


class Session:
    """One command's arguments plus its storage, opened lazily and closed at exit."""

    def __init__(self, args: argparse.Namespace) -> None:
        self.args = args
        self._db = self._cache = None

    def __enter__(self) -> Session:
        return self

    def __exit__(self, *exc) -> None:
        if self._db is not None:
            self._db.close()

    @property
    def db(self):
        """The results database, or None with ``--no-db``."""
        if self._db is None and not getattr(self.args, "no_db", False):
            from kernelo_b200.db import ResultsDB

            self._db = ResultsDB(self.args.db)
        return self._db

    @property
    def cache(self):
        """The tuned-config cache, or None with ``--no-cache``."""
        if self._cache is None and not getattr(self.args, "no_cache", False):
            from kernelo_b200.tuning.cache import ConfigCache

            self._cache = ConfigCache(self.args.cache)
        return self._cache

    def problem(self) -> Problem:
        return build_problem(self.args.operation, self.args)

    def header(self, problem: Problem) -> str:
        from kernelo_b200.runtime.env import capture_environment

        gpu = capture_environment().gpu_name or "none (CPU only)"
        names = "/".join(name for name, _ in problem.dims)
        sizes = " x ".join(str(size) for _, size in problem.dims)
        return f"GPU:    {gpu}\nShape:  {sizes}  ({names})\ndtype:  {problem.dtype_name.upper()}"


def rate(operator, problem: Problem, ms: float) -> tuple[str, float | None, float | None]:
    """The operator's figure of merit at ``ms``: text, TFLOP/s, GB/s."""
    from kernelo_b200.benchmark.metrics import gbps, tflops

    if operator.is_memory_bound():
        value = gbps(operator.bytes_moved(problem), ms)
        return f"{value:.1f} GB/s", None, value
    value = tflops(operator.flops(problem), ms)
    return f"{value:.1f} TFLOP/s", value, None


def implementations(operator, problem: Problem, inputs, config) -> dict[str, Callable[[], object]]:
    """Every label to compare: the operator's baselines and this library at ``config``."""
    labels = dict(operator.baselines(problem, inputs))
    labels["kernelforge"] = lambda: operator.run(config, *inputs)
    return labels


def gated_timings(session: Session, operator, problem: Problem, inputs, config, device):
    """(label, timing, verification) for every implementation that passes the
    gate against the reference, plus (label, message) for the others."""
    from kernelo_b200.benchmark.runner import benchmark
    from kernelo_b200.testing import exact_fp32_matmul, verify

    args = session.args
    with exact_fp32_matmul():
        reference = operator.reference(*inputs)
    passed, failed = [], []
    for label, call in implementations(operator, problem, inputs, config).items():
        try:
            check = verify(reference, call(), dtype=problem.dtype)
        except Exception as exc:  # noqa: BLE001 - a failing implementation is reported, not fatal
            failed.append((label, f"failed: {type(exc).__name__}"))
            continue
        if not check.passed:
            failed.append((label, f"INCORRECT: {check.reason}"))
            continue
        timing = benchmark(call, warmup=args.warmup, iterations=args.iterations, device=device,
                           flush_l2=not args.no_flush_l2)
        passed.append((label, timing, check))
    return passed, failed


# ------------------------------------------------------------------ commands
class Command:
    name = ""
    help = ""

    def configure(self, parser: argparse.ArgumentParser) -> None:
        """Add this command's arguments."""

    def run(self, session: Session) -> int:
        raise NotImplementedError


def _shape_flags(parser: argparse.ArgumentParser) -> None:
    group = parser.add_argument_group("shape", "dimensions for the selected operation; sensible defaults apply")
    group.add_argument("-m", "--m", type=int, help="GEMM rows of A (matmul, fused_linear, gemv)")
    group.add_argument("-n", "--n", type=int, help="GEMM columns of B")
    group.add_argument("-k", "--k", type=int, help="GEMM reduction size")
    group.add_argument("--rows", type=int, help="rows (rmsnorm, softmax)")
    group.add_argument("--cols", type=int, help="row width (rmsnorm, softmax)")


def _timing_flags(parser: argparse.ArgumentParser, *, warmup: int = 25, iterations: int = 200) -> None:
    parser.add_argument("--dtype", default="fp16", choices=SUPPORTED_DTYPES)
    parser.add_argument("--warmup", type=int, default=warmup)
    parser.add_argument("--iterations", type=int, default=iterations)
    parser.add_argument("--no-flush-l2", action="store_true",
                        help="do not flush L2 between iterations (inflates cache-resident problems)")


def _storage_flags(parser: argparse.ArgumentParser) -> None:
    from kernelo_b200.db import default_db_path
    from kernelo_b200.tuning.cache import default_cache_path

    parser.add_argument("--db", default=str(default_db_path()), help="results database path")
    parser.add_argument("--no-db", action="store_true", help="do not record results")
    parser.add_argument("--cache", default=str(default_cache_path()), help="config cache path")
    parser.add_argument("--no-cache", action="store_true", help="ignore and do not write the cache")


class EnvCommand(Command):
    name, help = "env", "print GPU, driver and library versions and device limits"

    def run(self, session: Session) -> int:
        from kernelo_b200.runtime.env import capture_environment, device_caps

        env = capture_environment()
        caps = device_caps()
        print(env.render())
        if env.gpu_name is None:
            print("\nNo CUDA device: kernels cannot run here; the tuning core and the B200 search spaces "
                  "can still be inspected (tune --explain).")
        print(heading("Device limits" + ("" if caps.measured else " (B200 target, no device attached)")))
        limits = {
            "SMs": caps.sm_count,
            "Shared memory per block (opt-in)": f"{caps.max_shared_memory_per_block // 1024} KiB",
            "Shared memory per SM": f"{caps.shared_memory_per_sm // 1024} KiB",
            "TMEM columns per SM": caps.tmem_columns_per_sm,
            "Registers per SM": caps.registers_per_sm,
            "Max threads per SM": caps.max_threads_per_sm,
            "L2 cache": f"{caps.l2_cache_bytes >> 20} MiB",
            "Cache key": caps.key,
        }
        pad = max(map(len, limits)) + 2
        for what, value in limits.items():
            print(f"{what.ljust(pad)}{value}")
        return 0


class TuneCommand(Command):
    name, help = "tune", "search configurations for one problem"

    def configure(self, parser):
        parser.add_argument("operation", choices=OPERATIONS)
        _shape_flags(parser)
        _timing_flags(parser)
        _storage_flags(parser)
        parser.add_argument("--max-candidates", type=int, help="override the candidate budget")
        parser.add_argument("--no-baselines", action="store_true", help="skip comparison baselines")
        parser.add_argument("--explain", action="store_true",
                            help="print the candidate-generation breakdown and exit without tuning")
        parser.add_argument("--resume", action="store_true",
                            help="reuse candidates the database already holds for this problem and device")

    def run(self, session: Session) -> int:
        args = session.args
        problem = session.problem()
        if args.explain:
            from kernelo_b200.runtime.env import device_caps
            from kernelo_b200.tuning.search import search_space

            space = search_space(args.operation, **({"max_candidates": args.max_candidates}
                                                    if args.max_candidates else {}))
            print(space.explain(problem, device_caps()))
            return 0
        from kernelo_b200.kernels import get_operator
        from kernelo_b200.tuning.tuner import Tuner

        if args.resume and args.no_db:
            raise ValueError("--resume reads the results database; drop --no-db")
        operator = get_operator(args.operation)
        print(session.header(problem) + "\n")
        tuner = Tuner(warmup=args.warmup, iterations=args.iterations, max_candidates=args.max_candidates,
                      measure_baselines=not args.no_baselines, flush_l2=not args.no_flush_l2, db=session.db,
                      cache=session.cache, log=print, resume=args.resume)
        result = tuner.tune(operator, problem)
        print(f"\nSearch space: {result.generated} grid points, {result.feasible} feasible, "
              f"{result.tested} measured in {result.elapsed_s:.1f}s")
        print(self.summary(result, operator))
        return 0 if result.best is not None else 1

    @staticmethod
    def summary(result, operator) -> str:
        from kernelo_b200.benchmark import metrics

        out = [heading("Best configuration")]
        best = result.best
        if best is None:
            out.append("No configuration passed verification.")
            out += [f"  {status}: {n}" for status, n in sorted(result.status_counts().items())]
            return "\n".join(out)
        out += [best.config.render(operator.config_order), heading("Performance")]
        times = Table("impl", "median ms", right=("median ms",))
        for label, timing in sorted([*result.baselines.items(), ("kernelforge", best.timing)],
                                    key=lambda item: item[1].median_ms):
            times.add(label, f"{timing.median_ms:.3f}")
        out.append(times.render())
        derived = Table("figure", "value", right=("value",))
        for label in ("torch_eager", "torch_compile", "cuda"):
            speedup = result.speedup_over(label)
            if speedup is not None:
                derived.add(f"speedup vs {label}", f"{speedup:.2f}x")
        if operator.is_memory_bound():
            derived.add("bandwidth", f"{result.gbps(best.median_ms):.1f} GB/s")
        else:
            derived.add("throughput", f"{result.tflops(best.median_ms):.1f} TFLOP/s")
        derived.add("arithmetic intensity",
                    f"{metrics.arithmetic_intensity(result.flops, result.bytes_moved):.1f} FLOP/byte")
        out += ["", derived.render()]
        return "\n".join(out)


class BenchmarkCommand(Command):
    name, help = "benchmark", "run a named workload suite"

    def configure(self, parser):
        from kernelo_b200.benchmark.workloads import SUITES

        parser.add_argument("operation", choices=OPERATIONS)
        parser.add_argument("--suite", default="sweep", choices=SUITES)
        _timing_flags(parser, iterations=100)
        _storage_flags(parser)

    def run(self, session: Session) -> int:
        from kernelo_b200.benchmark import workloads
        from kernelo_b200.db import Measurement
        from kernelo_b200.kernels import get_operator
        from kernelo_b200.runtime.dispatch import select_config
        from kernelo_b200.runtime.env import capture_environment, require_cuda

        args = session.args
        device = require_cuda()
        operator = get_operator(args.operation)
        env = capture_environment(device)
        db = session.db
        run_id = db.start_run(env, notes=f"benchmark:{args.suite}", version=__version__) if db else None
        print(env.render())
        print(heading(f"{args.operation} / {args.suite} / {args.dtype}"))
        table = Table("shape", "impl", "median ms", "p99 ms", "metric", right=("median ms", "p99 ms", "metric"))
        for problem in workloads.problems(args.operation, args.suite, args.dtype):
            inputs = operator.make_inputs(problem, device)
            config = select_config(operator, problem, cache=session.cache, device=device).config
            passed, failed = gated_timings(session, operator, problem, inputs, config, device)
            for label, message in failed:
                table.add(problem.shape_key, label, "", "", message)
            for label, timing, check in passed:
                text, tf, gb = rate(operator, problem, timing.median_ms)
                table.add(problem.shape_key, label, f"{timing.median_ms:.4f}", f"{timing.p99_ms:.4f}", text)
                if db is not None:
                    db.record(run_id, problem, Measurement(label, "ok", config if label == "kernelforge" else None,
                                                           check, timing, tf, gb))
        print(table.render())
        return 0


class CompareCommand(Command):
    name, help = "compare", "compare implementations at one shape, or a whole transformer block"

    def configure(self, parser):
        parser.add_argument("operation", choices=(*OPERATIONS, "transformer"))
        _shape_flags(parser)
        _timing_flags(parser, iterations=100)
        _storage_flags(parser)
        block = parser.add_argument_group("transformer", "block geometry for `compare transformer`")
        block.add_argument("--batch", type=int, default=1, help="transformer: batch size")
        block.add_argument("--seq", type=int, default=2048, help="transformer: sequence length")
        block.add_argument("--hidden", type=int, default=4096, help="transformer: hidden size")
        block.add_argument("--heads", type=int, default=32, help="transformer: attention heads")
        block.add_argument("--intermediate", type=int, default=11008, help="transformer: MLP intermediate size")

    def run(self, session: Session) -> int:
        if session.args.operation == "transformer":
            return self.transformer(session)
        from kernelo_b200.kernels import get_operator
        from kernelo_b200.runtime.dispatch import select_config
        from kernelo_b200.runtime.env import require_cuda

        device = require_cuda()
        operator = get_operator(session.args.operation)
        problem = session.problem()
        print(session.header(problem))
        inputs = operator.make_inputs(problem, device)
        selection = select_config(operator, problem, cache=session.cache, device=device)
        print(f"config: {selection.describe()}")
        print("        " + ", ".join(f"{k}={v}" for k, v in selection.config.as_dict().items()))
        passed, failed = gated_timings(session, operator, problem, inputs, selection.config, device)
        print(heading("Comparison"))
        for label, message in failed:
            print(f"{label}: {message}")
        passed.sort(key=lambda row: row[1].median_ms)
        eager = {label: t.median_ms for label, t, _ in passed}.get("torch_eager")
        table = Table("impl", "median ms", "p99 ms", "vs eager", "metric", "max err",
                      right=("median ms", "p99 ms", "vs eager", "metric", "max err"))
        for label, timing, check in passed:
            table.add(label, f"{timing.median_ms:.4f}", f"{timing.p99_ms:.4f}",
                      f"{eager / timing.median_ms:.2f}x" if eager else "-",
                      rate(operator, problem, timing.median_ms)[0], f"{check.error:.2e}")
        print(table.render())
        return 0

    @staticmethod
    def transformer(session: Session) -> int:
        from kernelo_b200.integration import BlockConfig, amdahl_breakdown
        from kernelo_b200.runtime.env import require_cuda

        args = session.args
        device = require_cuda()
        geometry = BlockConfig(hidden=args.hidden, heads=args.heads, intermediate=args.intermediate)
        print(f"Transformer block: hidden={geometry.hidden} heads={geometry.heads} "
              f"intermediate={geometry.intermediate} batch={args.batch} seq={args.seq} dtype={args.dtype}")
        breakdown = amdahl_breakdown(geometry, batch=args.batch, seq=args.seq, dtype=parse_dtype(args.dtype),
                                     device=device, warmup=args.warmup, iterations=args.iterations,
                                     cache=session.cache)
        print(heading("Block latency"))
        print(breakdown.render())
        print("\nOnly the two RMSNorms and the MLP up-projection + GELU are swapped; attention and the\n"
              "other projections are PyTorch in both, so the block speedup is bounded by the share of\n"
              "block time the swapped operators held.")
        return 0


def nsight_child_argv(args: argparse.Namespace) -> list[str]:
    """Arguments of the single-launch process that ncu profiles, rebuilt from
    the parsed arguments (shape flags given after ``--backend`` are kept); the
    cache is passed through so the child runs the parent's config."""
    child = ["profile", args.operation, "--dtype", args.dtype]
    for flag, dest in (("-m", "m"), ("-n", "n"), ("-k", "k"), ("--rows", "rows"), ("--cols", "cols")):
        value = getattr(args, dest)
        if value is not None:
            child += [flag, str(value)]
    child += ["--no-cache"] if args.no_cache else ["--cache", args.cache]
    return [*child, "--no-db", "--backend", "launch-once"]


class ProfileCommand(Command):
    name, help = "profile", "attribute time to kernels and counters"

    def configure(self, parser):
        from kernelo_b200.profiling.nsight import DEFAULT_SECTIONS, SECTIONS

        parser.add_argument("operation", choices=OPERATIONS)
        _shape_flags(parser)
        _timing_flags(parser, warmup=10, iterations=20)
        _storage_flags(parser)
        parser.add_argument("--backend", default="torch", choices=("torch", "nsight", "launch-once"),
                            help="torch: kernel attribution; nsight: hardware counters via ncu (clocks never "
                                 "locked); launch-once: a single launch, the ncu target")
        parser.add_argument("--sections", nargs="+", default=list(DEFAULT_SECTIONS), choices=sorted(SECTIONS),
                            help="Nsight Compute sections to collect")
        parser.add_argument("--report", help="write an .ncu-rep report to this path")

    def run(self, session: Session) -> int:
        args = session.args
        if args.backend == "nsight":
            from kernelo_b200.profiling import nsight

            if not nsight.ncu_available():
                print("ncu not found on PATH; install NVIDIA Nsight Compute.", file=sys.stderr)
                return 2
            capture = nsight.run(nsight.self_command(nsight_child_argv(args)), sections=tuple(args.sections),
                                 report_path=args.report, launch_count=1)
            print(capture.render())
            return 0 if capture.ok else 1
        import torch

        from kernelo_b200.kernels import get_operator
        from kernelo_b200.runtime.dispatch import select_config
        from kernelo_b200.runtime.env import require_cuda

        device = require_cuda()
        operator = get_operator(args.operation)
        problem = session.problem()
        inputs = operator.make_inputs(problem, device)
        config = select_config(operator, problem, cache=session.cache, device=device).config
        if args.backend == "launch-once":
            operator.run(config, *inputs)
            torch.cuda.synchronize()
            return 0
        from kernelo_b200.profiling import compare_launch_counts

        print(session.header(problem))
        print(heading("Kernel attribution"))
        for attribution in compare_launch_counts(implementations(operator, problem, inputs, config),
                                                 warmup=args.warmup, iterations=args.iterations):
            print(attribution.render() + "\n")
        return 0


class ReportCommand(Command):
    name, help = "report", "render tables from the results database"

    def configure(self, parser):
        _storage_flags(parser)
        parser.add_argument("--out", default="reports", help="output directory")

    def run(self, session: Session) -> int:
        from kernelo_b200.benchmark import report
        from kernelo_b200.db import ResultsDB

        path = Path(session.args.db)
        if not path.exists():
            print(f"no results database at {path}; run `python -m kernelo_b200 tune` first.", file=sys.stderr)
            return 2
        with ResultsDB(path) as db:
            n = db.counts()
            print(f"{n['results']} measurements across {n['problems']} problems and {n['runs']} runs")
            print(report.generate(db, session.args.out).render())
        return 0


class CacheCommand(Command):
    name, help = "cache", "inspect or clear the tuned-config cache"

    def configure(self, parser):
        parser.add_argument("cache_command", choices=("list", "clear"))
        _storage_flags(parser)

    def run(self, session: Session) -> int:
        from kernelo_b200.tuning.cache import ConfigCache

        cache = ConfigCache(session.args.cache)
        if session.args.cache_command == "clear":
            print(f"removed {cache.clear()} cached configuration(s) from {cache.path}")
            return 0
        entries = cache.entries()
        print(f"{cache.path}: {len(entries)} entry(ies)")
        print("\n".join(f"  {e.describe()}" for e in entries))
        return 0


COMMANDS: tuple[Command, ...] = (EnvCommand(), TuneCommand(), BenchmarkCommand(), CompareCommand(),
                                 ProfileCommand(), ReportCommand(), CacheCommand())


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="python -m kernelo_b200",
                                     description="B200-native KernelForge hot path: tune, benchmark, compare, "
                                                 "profile and report.")
    parser.add_argument("--version", action="version", version=f"kernelo_b200 {__version__}")
    sub = parser.add_subparsers(dest="command", required=True)
    for command in COMMANDS:
        command.configure(sub.add_parser(command.name, help=command.help))
    return parser


def main(argv: list[str] | None = None) -> int:
    args = build_parser().parse_args(argv)
    command = next(c for c in COMMANDS if c.name == args.command)
    try:
        with Session(args) as session:
            return command.run(session)
    except KeyboardInterrupt:
        print("\ninterrupted", file=sys.stderr)
        return 130
    except (RuntimeError, ValueError) as exc:
        print(f"error: {exc}", file=sys.stderr)
        return 1
