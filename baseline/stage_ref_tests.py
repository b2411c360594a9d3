"""Stage the reference's own GPU tests to run on this library (drop-in check).

The reference drives its GPU environment through the ``junqi_cuda`` module.
This script builds, under ``baseline/_ref/dropin`` (git-ignored), a copy of
the reference's Python packages and of its tests that use that module,
with ``junqi_rl/junqi_cuda.py`` replaced by the one-file shim a maintainer
would add (it routes ``import junqi_cuda`` to ``junqi_b200.junqi_cuda``).
The reference's compiled extension is not copied, so every test there runs
on this library's kernels.  Run on a GPU box from the repository root::

    python baseline/stage_ref_tests.py <reference checkout>      # where the checkout exists
    cd baseline/_ref/dropin && python -m pytest -q -p no:cacheprovider tests

Nothing is written into the reference checkout.
"""
from __future__ import annotations

import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
OUT = HERE / "_ref" / "dropin"
# the reference's tests that exercise junqi_cuda (directly or through GpuRollout / GpuWorld / env_gpu)
TESTS = ["test_gpu_step_batch.py", "test_gpu_csr_mask.py", "test_gpu_obs_parity.py",
         "test_gpu_combat_memory_parity.py", "test_gpu_legal_lite.py", "test_legal_actions_gpu.py",
         "test_legal_actions_gpu_stress.py", "test_gpu_engineer_adversarial.py", "test_gpu_rollout.py",
         "test_gpu_world.py", "test_env_gpu_cpu.py", "test_compact_rollout_history.py",
         "test_initial_setup_pool_reset.py", "test_torch_zero_copy.py", "test_pool_upload.py",
         "test_gpu_collector.py", "test_gpu_collector_e2e.py"]

SHIM = '''"""Route ``import junqi_cuda`` to the B200 library (junqi_b200.junqi_cuda)."""
import sys
sys.path.insert(0, {repo!r})
from junqi_b200 import junqi_cuda as _impl
sys.modules[__name__] = _impl
'''


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: python baseline/stage_ref_tests.py <reference checkout>")
    ref = Path(sys.argv[1]).resolve()
    if OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir(parents=True)
    skip = shutil.ignore_patterns("*.so", "__pycache__", "build")
    for pkg in ("junqi_core", "junqi_rl", "legacy_common"):
        if (ref / pkg).exists():
            shutil.copytree(ref / pkg, OUT / pkg, ignore=skip)
    for f in ("conftest.py", "pyproject.toml"):
        shutil.copy(ref / f, OUT / f)
    (OUT / "tests").mkdir()
    for f in ["__init__.py", "conftest.py"] + TESTS:
        if (ref / "tests" / f).exists():
            shutil.copy(ref / "tests" / f, OUT / "tests" / f)
    if (ref / "tests" / "golden").exists():
        shutil.copytree(ref / "tests" / "golden", OUT / "tests" / "golden")
    # the relative path keeps the staged tree valid wherever the repository is checked out
    (OUT / "junqi_rl" / "junqi_cuda.py").write_text(
        SHIM.replace("{repo!r}", "__import__('os').path.abspath(__import__('os').path.join("
                                 "__import__('os').path.dirname(__file__), '..', '..', '..', '..'))"))
    print("staged", len(TESTS), "test files under", OUT)


if __name__ == "__main__":
    main()
