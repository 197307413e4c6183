"""Builds the reference's own CUDA selective-scan module into oracle/_ref/.

TEST INFRASTRUCTURE ONLY: the fp16 comparator of the forward parity tests. Nothing in the
product path imports it.

The reference keeps its CUDA kernels and pybind host functions as two string constants,
``cuda_source`` and ``cpp_source``, in mamba_windows_cuda/mamba_cuda.py, and JIT-compiles
them with torch.utils.cpp_extension.load_inline under MSVC-only host flags
(mamba_cuda.py:835-872). This recipe reads the two strings from the reference checkout with
``ast`` (the reference module is never imported or executed), and compiles them unchanged
with the reference's own device flags (-O3 --use_fast_math, its default
MAMBA_CUDA_USE_FAST_MATH=1) for sm_100a, without the MSVC host flags. The sources and the
built extension stay in oracle/_ref/ (git-ignored); the built .so travels to the GPU box.

Usage: python oracle/build_ref.py [REFERENCE_ROOT]   (or set MWC_REFERENCE_ROOT)
Without a reference checkout it does nothing (the GPU box uses the prebuilt module).
"""
from __future__ import annotations

import ast
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "mwc_reference_scan"
FUNCTIONS = ["selective_scan_cuda_forward", "selective_scan_cuda_forward_with_state",
             "selective_scan_cuda_backward", "selective_scan_cuda_forward_store",
             "selective_scan_cuda_backward_direct"]


def _sources(ref_root: str):
    path = os.path.join(ref_root, "mamba_windows_cuda", "mamba_cuda.py")
    tree = ast.parse(open(path, encoding="utf-8").read(), filename=path)
    found = {}
    for node in tree.body:
        if isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Name):
            name = node.targets[0].id
            if name in ("cuda_source", "cpp_source") and isinstance(node.value, ast.Constant):
                found[name] = node.value.value
    if set(found) != {"cuda_source", "cpp_source"}:
        raise RuntimeError(f"cuda_source / cpp_source not found in {path}")
    return found["cpp_source"], found["cuda_source"]


def built_path():
    """Path of the built extension module, or None."""
    d = os.path.join(OUT, "build")
    if not os.path.isdir(d):
        return None
    for f in sorted(os.listdir(d)):
        if f.startswith(NAME) and f.endswith(".so"):
            return os.path.join(d, f)
    return None


def load():
    """Import the prebuilt reference module (None when it was not built)."""
    path = built_path()
    if path is None:
        return None
    import torch  # noqa: F401  (the extension links against libtorch)
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def build(ref_root: str | None = None) -> str | None:
    ref_root = ref_root or os.environ.get("MWC_REFERENCE_ROOT")
    if not ref_root or not os.path.isfile(os.path.join(ref_root, "mamba_windows_cuda", "mamba_cuda.py")):
        return built_path()
    cpp, cuda = _sources(ref_root)
    os.makedirs(os.path.join(OUT, "build"), exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load_inline
    load_inline(name=NAME, cpp_sources=cpp, cuda_sources=cuda, functions=FUNCTIONS,
                build_directory=os.path.join(OUT, "build"), verbose=False,
                extra_cuda_cflags=["-O3", "--use_fast_math",
                                   "-gencode=arch=compute_100a,code=sm_100a"])
    return built_path()


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None))
