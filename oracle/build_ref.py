"""Builds the reference's own native score kernel as a checker — TEST
INFRASTRUCTURE ONLY.

The reference's only compiled source for the hot path is
modules/kvr_cuda.cu (a torch extension the reference JIT-builds with
torch.utils.cpp_extension.load, modules/kvr_cuda.py:7-17).  This recipe
compiles that file, unmodified and from where it lies in the reference
checkout, with the same torch extension machinery, for sm_100a, into
oracle/_ref/ (git-ignored; the built module travels with the repository
snapshot to the GPU box).  Only tests import the result, to check
kvr_compute_scores bit-for-bit against the reference kernel.

    python oracle/build_ref.py <path to the reference checkout>
"""
import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "kvr_cuda_ref"


def built_module_path():
    hits = glob.glob(os.path.join(OUT, NAME + "*.so"))
    return hits[0] if hits else None


def build(reference_root, verbose=False):
    src = os.path.join(reference_root, "modules", "kvr_cuda.cu")
    if not os.path.exists(src):
        raise FileNotFoundError(src)
    os.makedirs(OUT, exist_ok=True)
    so = os.path.join(OUT, NAME + ".so")
    if os.path.exists(so) and os.path.getmtime(so) >= os.path.getmtime(src):
        return so
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    from torch.utils.cpp_extension import load

    # builds OUT/kvr_cuda_ref.so; loading it needs no GPU
    load(name=NAME, sources=[src], build_directory=OUT, verbose=verbose, is_python_module=True)
    return so


def load_module():
    """Import the built reference extension (None if it was not built)."""
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401 - the extension links against libtorch

    path = built_module_path()
    if path is None:
        return None
    loader = importlib.machinery.ExtensionFileLoader(NAME, path)
    spec = importlib.util.spec_from_file_location(NAME, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python oracle/build_ref.py <path to the reference checkout>")
    print(build(sys.argv[1], verbose=True))
