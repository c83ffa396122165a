"""Build the packmla CUDA extension in-tree for sm_100a only.

    python setup.py build_ext --inplace

The extension is compiled for `sm_100a` with explicit -gencode flags; no other
architecture is targeted (tcgen05 / TMEM instructions exist only there).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/torch_ops.cpp"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("PACKMLA_PTXAS_VERBOSE") else "-O3",
]


class _RecordingBuild(BuildExtension.with_options(use_ninja=True)):
    """Records the digest of the built sources beside the library (packmla/_C.sources.json)."""

    def run(self):
        super().run()
        import importlib.util

        spec = importlib.util.spec_from_file_location("source_digest",
                                                      os.path.join(ROOT, "packmla", "utils", "source_digest.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.write_record(ROOT)


setup(
    name="packmla",
    version="0.1.0",
    packages=["packmla"],
    ext_modules=[
        CUDAExtension(
            name="packmla._C",
            sources=SOURCES,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            libraries=["cuda"],
        )
    ],
    cmdclass={"build_ext": _RecordingBuild},
)
