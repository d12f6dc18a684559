"""`openquant` command line (openquant/cli.py:6-92): --version, cpu, gpu, tune,
report.  `gpu` and `tune` run the B200 kernels (fused_benchmark, autotune);
`cpu` and `report` keep the reference's reports, computed on the GPU."""
import argparse
import json
from pathlib import Path

__all__ = ["main"]


def main(argv=None):
    parser = argparse.ArgumentParser(prog="openquant", description="OpenQuant AI optimization toolkit (B200 build)")
    parser.add_argument("--version", action="version", version="OpenQuant 0.5.0 (openquant_b200 0.1.0, sm_100a)")
    commands = parser.add_subparsers(dest="command")
    cpu = commands.add_parser("cpu")
    cpu.add_argument("--rows", type=int, default=1024)
    cpu.add_argument("--cols", type=int, default=1024)
    commands.add_parser("gpu")
    tune = commands.add_parser("tune")
    tune.add_argument("--output", default=None)
    tune.add_argument("--quick", action="store_true")
    report = commands.add_parser("report", help="Save a reproducible quantization report")
    report.add_argument("--rows", type=int, default=1024)
    report.add_argument("--cols", type=int, default=1024)
    report.add_argument("--seed", type=int, default=42)
    report.add_argument("--group-size", type=int, default=32)
    report.add_argument("--output", default="reports/openquant_cpu.json")
    args = parser.parse_args(argv)

    if args.command == "cpu":
        if args.rows <= 0 or args.cols <= 0:
            parser.error("Dimensions must be positive")
        from .benchmark import benchmark

        benchmark(args.rows, args.cols)
    elif args.command == "gpu":
        from .fused_benchmark import main as run

        run()
    elif args.command == "tune":
        from .autotune import main as run

        targs = (["--output", args.output] if args.output else []) + (["--quick"] if args.quick else [])
        run(targs)
    elif args.command == "report":
        from .report import make_cpu_report

        try:
            data = make_cpu_report(rows=args.rows, cols=args.cols, seed=args.seed, group_size=args.group_size)
        except ValueError as exc:
            parser.error(str(exc))
        output = Path(args.output)
        output.parent.mkdir(parents=True, exist_ok=True)
        output.write_text(json.dumps(data, indent=2, allow_nan=False) + "\n", encoding="utf-8")
        print("Report saved:", output.resolve())
        for name, metrics in data["formats"].items():
            print(f"{name:<16}{metrics['memory_reduction_pct']:>8.2f}% saved  error: "
                  f"{metrics['relative_weight_error_pct']:.3f}%")
    else:
        parser.print_help()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
