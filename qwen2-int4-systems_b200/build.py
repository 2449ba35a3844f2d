"""Build ``libqi4_b200.so`` (the C-ABI backend) in-tree with nvcc for sm_100a.

    python -m <package>.build          # or: python qwen2-int4-systems_b200/build.py

Objects go to ``_build/`` at the repository root; the shared library is
written next to this file so that it travels with the source tree. Rebuilds
only what changed (source or header newer than its object).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libqi4_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden", "-Xptxas", "-v",
    "-I", str(ROOT / "include"), "-I", str(CSRC),
    "--expt-relaxed-constexpr",
]
# Only the extern "C" entry points are exported.
EXPORTS = [
    "qi4_w4g64_linear", "qi4_w4g64_linear_ex", "qi4_w4g64_dequant_f32",
    "qi4_w4_unpack", "qi4_w4g64_linear_f32_noalloc", "qi4_gemv_plan_override", "qi4_gemv_mma_plan_override", "qi4_gemm_tc_plan_override", "qi4_gemv_mma_plan", "qi4_w4g64_linear_multi", "qi4_w4g64_gate_up_silu", "qi4_device_status", "qi4_selftest_bounded_wait",
    "qi4_chain_create", "qi4_chain_run", "qi4_chain_info", "qi4_chain_destroy", "qi4_gqa_decode_attention", "qi4_bf16_gemv_argmax", "qi4_add_rmsnorm",
    "qi4_w4g64_linear_multi_norm", "qi4_w4g64_gate_up_silu_norm", "qi4_gqa_decode_attention_workspace", "qi4_gqa_decode_attention_ex", "qi4_bf16_gemv_argmax_ws", "qi4_bf16_argmax_rows", "qi4_w4g64_gate_up_silu_scatter", "qi4_peer_flag_wait", "qi4_ipc_alloc", "qi4_ipc_open", "qi4_ipc_close", "qi4_ipc_free", "qi4_last_error", "qi4_version",
]


def nvcc() -> str:
    for cand in (os.environ.get("CUDA_HOME", ""), "/usr/local/cuda"):
        if cand and (Path(cand) / "bin" / "nvcc").exists():
            return str(Path(cand) / "bin" / "nvcc")
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; the B200 backend needs the CUDA toolkit to build")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _compile(src: Path, obj: Path, log: Path) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}{proc.stderr}")


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs = []
    objects = []
    for src in _sources():
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        stale = (force or not obj.exists()
                 or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header))
        if stale:
            jobs.append((src, obj, BUILD / (src.stem + ".log")))
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as pool:
            list(pool.map(lambda j: _compile(*j), jobs))
        if verbose:
            for _, _, log in jobs:
                print(log.read_text())
    link_needed = force or jobs or not LIB.exists() or any(
        o.stat().st_mtime > LIB.stat().st_mtime for o in objects)
    if link_needed:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp),
               *map(str, objects), "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}{proc.stderr}")
        os.replace(tmp, LIB)
    return LIB


REFERENCE_SRC = Path("/root/reference")
HARNESS = ROOT / "baseline" / "_ref"


def install_reference_harness(source: Path = REFERENCE_SRC, force: bool = False) -> Path | None:
    """Install the reference project's pure-Python package into ``baseline/_ref``.

    The model-level GPU tests and the bench's decode section run the
    reference's own ``QwenInt4ForCausalLM`` and generation loop unchanged on
    the ``b200`` backend; this puts that code where ``qwen2.reference_package``
    looks for it, so that it travels with the tree to a machine without the
    reference checkout. ``pip install --no-deps --target`` from a temporary
    copy (the build writes into its source tree). Returns the target, or None
    when no reference checkout is present (the files already installed are
    then used as they are)."""
    import tempfile

    if not force and (HARNESS / "qwen_int4" / "model.py").exists():
        return HARNESS
    if not (source / "src" / "qwen_int4").is_dir():
        return None
    with tempfile.TemporaryDirectory() as tmp:
        copy = Path(tmp) / "reference"
        shutil.copytree(source, copy, ignore=shutil.ignore_patterns(".git", "__pycache__"))
        staging = HARNESS.with_name("_ref.tmp")
        shutil.rmtree(staging, ignore_errors=True)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", str(staging), "-q", str(copy)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"reference harness install failed:\n{proc.stdout}{proc.stderr}")
    shutil.rmtree(HARNESS, ignore_errors=True)
    os.replace(staging, HARNESS)
    return HARNESS


def binding_path() -> Path:
    import sysconfig
    return PKG / ("_qi4_torch" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_binding(force: bool = False) -> Path:
    """Compile csrc/torch_binding.cpp (the C++ fast path of the Python
    QuantLinear call) against this interpreter's torch and libqi4_b200.so,
    in-tree next to the library. Rebuilt when the source, the C header or the
    library is newer than the module."""
    import sysconfig

    import torch

    src = CSRC / "torch_binding.cpp"
    out = binding_path()
    deps = [src, ROOT / "include" / "qi4_b200.h", LIB]
    if not force and out.exists() and out.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return out
    torch_dir = Path(torch.__file__).resolve().parent
    cuda_home = Path(nvcc()).resolve().parent.parent
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [shutil.which("g++") or "g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_qi4_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-I", str(torch_dir / "include"), "-I", str(torch_dir / "include" / "torch" / "csrc" / "api" / "include"),
           "-I", sysconfig.get_paths()["include"], "-I", str(cuda_home / "include"), "-I", str(ROOT / "include"),
           str(src), "-o", str(out) + ".tmp",
           "-L", str(torch_dir / "lib"), "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10", "-lc10_cuda",
           "-L", str(PKG), "-lqi4_b200", "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + str(torch_dir / "lib")]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    (BUILD / "torch_binding.log").write_text(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
    if proc.returncode != 0:
        raise RuntimeError(f"torch binding build failed:\n{proc.stderr[-4000:]}")
    os.replace(str(out) + ".tmp", out)
    return out


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
    print(build_torch_binding(force="--force" in sys.argv))
