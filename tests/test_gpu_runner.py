"""The KernelBench-style runner (pla_b200.runner) drives the drop-in modules
against reference-shaped problem files, as run_generated_presburger_triton.py
drives generated kernels."""
import json
import os

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


@pytest.mark.parametrize("problem,kernel", [
    ("stencil_problem.py", "pla_b200/stencil.py"),
    ("depthwise_problem.py", "pla_b200/depthwise.py"),
])
def test_runner_checks_and_times(problem, kernel, tmp_path):
    from pla_b200 import runner

    out = tmp_path / "r.json"
    rc = runner.main(["--ref-arch-src-path", os.path.join(HERE, "problems", problem),
                      "--kernel-src-path", os.path.join(ROOT, kernel), "--result-json", str(out),
                      "--iters", "5", "--warmup", "2"])
    res = json.loads(out.read_text())
    assert rc == 0 and res["compiled"] and res["correctness"], res
    assert res["runtime_ms"] > 0 and res["ref_eager_ms"] > 0
    assert res["max_abs_err"] < 1e-5
