"""KernelBench-style check-and-time runner for a ``ModelNew`` file.

Stands in for the ``scripts.run_and_check.main`` call that
``run_generated_presburger_triton.py:72`` makes (KernelBench's harness is not
part of the reference snapshot).  Same CLI as the reference runner
(``run_generated_presburger_triton.py:81-112``):

    python -m pla_b200.runner --ref-arch-src-path <Model file> \\
        --kernel-src-path <ModelNew file> [--backend cuda] [--result-json out.json]

Steps, as the reference harness reports them (``:94-112``):
1. import both files; build ``Model(*get_init_inputs())`` on the CPU and
   ``ModelNew(*get_init_inputs())``; load the reference's state dict into the
   new model (the parameter names are the same by contract); move to CUDA;
2. correctness: ``--trials`` seeded draws of ``get_inputs()``; the reference
   module runs on the CPU (its own PyTorch path), the new one on the GPU;
   outputs must agree within ``--atol/--rtol`` (defaults 1e-5 fp32);
3. timing: CUDA events around ``--iters`` calls of each (eager reference on the
   GPU too, as KernelBench times it), after ``--warmup`` calls.

Writes ``{"compiled", "correctness", "runtime_ms", "ref_eager_ms",
"ref_compile_ms", "max_abs_err"}`` (``ref_compile_ms`` is null: no
``torch.compile`` run here).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys
from pathlib import Path

import torch


def _load(path: str, name: str):
    path = str(Path(path).resolve())
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _time(fn, inputs, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn(*inputs)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn(*inputs)
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def run_and_check(ref_path: str, kernel_path: str, trials: int = 3, iters: int = 20, warmup: int = 3,
                  atol: float = 1e-5, rtol: float = 1e-5, seed: int = 0, input_scale: float | None = None) -> dict:
    ref_mod = _load(ref_path, "pla_runner_ref")
    new_mod = _load(kernel_path, "pla_runner_new")
    init = ref_mod.get_init_inputs()
    result = {"compiled": False, "correctness": False, "runtime_ms": None, "ref_eager_ms": None,
              "ref_compile_ms": None, "max_abs_err": None}
    torch.manual_seed(seed)
    ref = ref_mod.Model(*init).eval()
    try:
        new = new_mod.ModelNew(*init).eval()
        new.load_state_dict(ref.state_dict())
        new = new.cuda()
        result["compiled"] = True
    except Exception as exc:  # noqa: BLE001 - reported, like the harness does
        result["error"] = f"{type(exc).__name__}: {exc}"
        return result
    max_err = 0.0
    ok = True
    inputs = None
    with torch.no_grad():
        for t in range(trials):
            torch.manual_seed(seed + t)
            inputs = ref_mod.get_inputs()
            if input_scale is not None:
                inputs = [x * input_scale for x in inputs]
            want = ref(*inputs)
            got = new(*[x.cuda() for x in inputs]).cpu()
            err = (got.double() - want.double()).abs().max().item() if got.numel() else 0.0
            max_err = max(max_err, err)
            ok = ok and got.shape == want.shape and torch.allclose(got, want, atol=atol, rtol=rtol)
        result["correctness"] = bool(ok)
        result["max_abs_err"] = max_err
        dev_inputs = [x.cuda() for x in inputs]
        result["runtime_ms"] = _time(new, dev_inputs, iters, warmup)
        ref_gpu = ref.cuda()
        result["ref_eager_ms"] = _time(ref_gpu, dev_inputs, iters, warmup)
    return result


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ref-arch-src-path", "--ref_arch_src_path", required=True)
    ap.add_argument("--kernel-src-path", "--kernel_src_path", required=True)
    ap.add_argument("--backend", choices=("triton", "cuda"), default="cuda",
                    help="accepted for CLI compatibility; the kernels here are CUDA")
    ap.add_argument("--result-json", type=Path)
    ap.add_argument("--trials", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--atol", type=float, default=1e-5)
    ap.add_argument("--rtol", type=float, default=1e-5)
    args = ap.parse_args(argv)
    res = run_and_check(args.ref_arch_src_path, args.kernel_src_path, args.trials, args.iters, args.warmup,
                        args.atol, args.rtol)
    for k in ("correctness", "runtime_ms", "ref_eager_ms", "ref_compile_ms"):
        print(f"{k}: {res[k]}")
    if args.result_json:
        args.result_json.write_text(json.dumps(res, indent=2) + "\n")
    return 0 if res["correctness"] else 1


if __name__ == "__main__":
    sys.exit(main())
