"""Run the CPU test suite against a sanitizer build of the C++ serving runtime.

    python -m sparkpipe_rs_b200.utils.sanitize --mode address   # ASan + UBSan
    python -m sparkpipe_rs_b200.utils.sanitize --mode thread    # TSan

The host runtime extension (`_sp_core`: scheduler, prefix cache, gateway with its
epoll thread, NVMe tier workers, KV store worker, multi-lane fabric transfers, rank
daemon, ...) is rebuilt with the sanitizer into its own directory
(SPARKPIPE_SANITIZE selects it, see _ext.py), then pytest runs the CPU tests with the
sanitizer runtime preloaded into the interpreter, so every instrumented access in
the extension is checked. The interpreter and torch are not instrumented: memory
errors and races are reported for the framework's own C++ code only. Leak checking
is off (the interpreter keeps its allocations until exit). A report fails the run;
the exit code is pytest's, or the sanitizer's on a report that aborts the process.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


def _lib(name: str) -> str:
    path = subprocess.run(["g++", f"-print-file-name={name}"], capture_output=True, text=True, check=True).stdout.strip()
    if not os.path.isabs(path) or not os.path.exists(path):
        raise RuntimeError(f"{name} not found")
    return os.path.realpath(path)


def runtime_library(mode: str) -> str:
    """The sanitizer runtime, then libstdc++: the runtime's C++ exception interceptor
    binds the real __cxa_throw when it starts, so libstdc++ must already be loaded."""
    return _lib("libasan.so" if mode == "address" else "libtsan.so") + " " + _lib("libstdc++.so.6")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["address", "thread"], default="address")
    ap.add_argument("--log", default="", help="also write the combined output here")
    ap.add_argument("pytest_args", nargs="*", help="extra pytest arguments (default: the CPU suite)")
    args = ap.parse_args()

    env = dict(os.environ)
    env["SPARKPIPE_SANITIZE"] = args.mode
    env["LD_PRELOAD"] = runtime_library(args.mode)
    if args.mode == "address":
        env["ASAN_OPTIONS"] = "detect_leaks=0:halt_on_error=1:exitcode=86:log_to_stderr=1"
        env["UBSAN_OPTIONS"] = "print_stacktrace=1:halt_on_error=1:exitcode=87"
    else:
        # torch's CPU kernels run on OpenMP threads that libgomp creates without TSan's
        # knowledge: one OpenMP thread, and races inside torch / libgomp are not reported.
        # The framework's own threads and the calls of _sp_core stay checked.
        sup = Path(os.environ.get("TMPDIR", "/tmp")) / "sparkpipe_tsan.supp"
        sup.write_text("race:libtorch_cpu.so\nrace:libgomp.so\ncalled_from_lib:libgomp.so\n"
                       )
        env["OMP_NUM_THREADS"] = "1"
        env["TSAN_OPTIONS"] = (f"halt_on_error=1:exitcode=88:report_signal_unsafe=0:second_deadlock_stack=1:"
                               f"suppressions={sup}")
    # build and import the instrumented extension first (the import needs the runtime
    # preloaded; the compiler children inherit it, which only slows them down)
    subprocess.run([sys.executable, "-c", "from sparkpipe_rs_b200 import _ext; _ext.build_all()"], cwd=ROOT, env=env,
                   check=True, stdout=subprocess.DEVNULL)
    cmd = [sys.executable, "-m", "pytest", "tests", "-q", "-m", "not gpu", "-p", "no:cacheprovider"]
    cmd += args.pytest_args
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    out = proc.stdout + proc.stderr
    header = (f"sanitizer run: mode={args.mode} preload={env['LD_PRELOAD']}\n"
              f"command: SPARKPIPE_SANITIZE={args.mode} LD_PRELOAD=<runtime> {' '.join(cmd[1:])}\n"
              f"exit code: {proc.returncode}\n\n")
    if args.log:
        Path(args.log).write_text(header + out)
    sys.stdout.write(header + out[-4000:])
    return proc.returncode


if __name__ == "__main__":
    sys.exit(main())
