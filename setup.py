"""Build the in-tree sm_100a extension: ``python setup.py build_ext --inplace``.

Produces ``afd_plugin_b200/_C*.so`` (loaded with ``torch.ops.load_library``).
Kernels are compiled for sm_100a only (tcgen05 / TMA code paths).
"""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("afd_plugin_b200", "ops", "csrc")


def _nccl_dirs():
    """NCCL headers / library matching the one PyTorch loads (the nvidia-nccl wheel)."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is not None and spec.submodule_search_locations:
        base = list(spec.submodule_search_locations)[0]
        return [os.path.join(base, "include")], [os.path.join(base, "lib")]
    return [], []


NCCL_INC, NCCL_LIB = _nccl_dirs()
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
DEBUG = os.environ.get("AFD_B200_KERNEL_DEBUG", "") in ("1", "true", "on")

nvcc_flags = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("AFD_B200_PTXAS_VERBOSE") else "-Xptxas=-O3",
] + (["-DAFD_KERNEL_DEBUG=1"] if DEBUG else [])

setup(
    name="afd_plugin_b200",
    version="0.1.0",
    packages=find_packages(include=["afd_plugin_b200", "afd_plugin_b200.*"]),
    ext_modules=[
        CUDAExtension(
            name="afd_plugin_b200._C",
            sources=sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp"))),
            include_dirs=[os.path.join(ROOT, CSRC)] + NCCL_INC,
            library_dirs=NCCL_LIB,
            # libnccl.so.2 is the library PyTorch itself loads (resolved by soname at load time)
            extra_link_args=[f"-Wl,-rpath,{d}" for d in NCCL_LIB] + (["-l:libnccl.so.2"] if NCCL_LIB else ["-lnccl"]),
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"vllm.general_plugins": ["afd = afd_plugin_b200:register_afd"],
                  "console_scripts": ["afd-b200 = afd_plugin_b200.__main__:main"]},
)
