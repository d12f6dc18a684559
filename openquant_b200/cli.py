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
    report.add_argument("--rows", type=int, default=None)
    report.add_argument("--cols", type=int, default=None)
    report.add_argument("--seed", type=int, default=42)
    report.add_argument("--group-size", type=int, default=None)
    report.add_argument("--output", default=None)
    report.add_argument("--gpu", action="store_true",
                        help="schema 2: add GPU timings of each format's kernels (default 4096 x 4096, group 128)")
    report.add_argument("--batch", type=int, default=1, help="activation rows for the fused products (--gpu)")
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
        from .report import make_cpu_report, make_gpu_report

        dflt = (4096, 4096, 128) if args.gpu else (1024, 1024, 32)
        rows = args.rows if args.rows is not None else dflt[0]
        cols = args.cols if args.cols is not None else dflt[1]
        group = args.group_size if args.group_size is not None else dflt[2]
        try:
            if args.gpu:
                data = make_gpu_report(rows=rows, cols=cols, seed=args.seed, group_size=group, batch=args.batch)
            else:
                data = make_cpu_report(rows=rows, cols=cols, seed=args.seed, group_size=group)
        except ValueError as exc:
            parser.error(str(exc))
        output = Path(args.output or ("reports/openquant_gpu.json" if args.gpu else "reports/openquant_cpu.json"))
        output.parent.mkdir(parents=True, exist_ok=True)
        output.write_text(json.dumps(data, indent=2, allow_nan=False) + "\n", encoding="utf-8")
        print("Report saved:", output.resolve())
        for name, metrics in data["formats"].items():
            print(f"{name:<16}{metrics['memory_reduction_pct']:>8.2f}% saved  error: "
                  f"{metrics['relative_weight_error_pct']:.3f}%")
        for name, kernels in data.get("gpu", {}).get("formats", {}).items():
            for kname, k in kernels.items():
                print(f"{name:<16}{kname:<16}{k['time_us']:>10.2f} us {k['GB_per_s']:>10.1f} GB/s")
    else:
        parser.print_help()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
