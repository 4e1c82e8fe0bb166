"""The drop-in boundary against the reference engine itself.

aethermind_b200/reference_plugin/cuda_backend_plugin.cpp is a CUDA backend
for the reference (fengjiran/AetherMind), compiled against its public headers:
kernels registered with its AM_REGISTER_KERNEL under kCUDA selectors, a
Backend and a BackendFactory for RuntimeBuilder::RegisterBackendFactory.
plugin_check (same folder) drives the reference's own RuntimeBuilder,
ExecutionPlanBuilder and Executor, compiled from its sources into
oracle/_ref/libam_ref.so, with that plugin:

  * resolve (CPU): a plan of kCUDA RmsNorm / Add nodes resolves the plugin's
    kernels through the reference's registry and planner; an unregistered
    kCUDA selector fails with the registry's NOT_FOUND;
  * execute (GPU): the plan runs through Executor::Execute on device tensors
    and reproduces the reference's RMSNorm unit-test golden values
    (tests/unit/backend/cpu/kernels/test_cpu_rmsnorm_kernel.cpp:65-89,
    126-129) and a bit-exact bf16 Add.

The binaries are built by __graft_entry__.build() where the reference
sources exist (oracle/_ref/ travels with the repository to the GPU box).
"""
import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CHECK = ROOT / "oracle" / "_ref" / "plugin" / "plugin_check"
REF_ROOT = Path(os.environ.get("AETHERMIND_REF_ROOT") or ROOT.parent / "reference")


def _ensure_built():
    if (REF_ROOT / "include").exists() and (ROOT / "oracle" / "_ref" / "libam_ref.so").exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "aethermind_b200" / "reference_plugin"),
                        f"REF_ROOT={REF_ROOT}"], check=True, capture_output=True)
    if not CHECK.exists():
        pytest.skip("the reference plugin builds only where the reference sources are present")


def _run(mode):
    r = subprocess.run([str(CHECK), mode], capture_output=True, text=True, timeout=120)
    return r.returncode, r.stdout + r.stderr


def test_plugin_kernels_resolve_through_reference_planner(built_lib):
    _ensure_built()
    rc, out = _run("resolve")
    assert rc == 0, out
    assert "step 0: aethermind_b200::rmsnorm_cuda_f32" in out
    assert "step 2: aethermind_b200::add_cuda_bf16" in out
    assert "NOT_FOUND" in out


@pytest.mark.gpu
def test_plugin_runs_reference_executor_on_gpu(built_lib):
    if not CHECK.exists():
        pytest.skip("plugin_check not built (needs the reference sources at build time)")
    rc, out = _run("execute")
    assert rc == 0, out
    assert "rmsnorm:" in out and out.rstrip().endswith("OK"), out
