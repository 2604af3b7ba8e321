"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Produces ``vllm_neuron_b200/_C*.so`` (every kernel, compiled only for
``arch=compute_100a,code=sm_100a``) next to the Python package, so it travels with
the source tree.
"""

import glob
import os

from setuptools import find_packages, setup

os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"  # keep torch from adding other targets
from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("vllm_neuron_b200", "csrc")
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
]

setup(
    name="vllm_neuron_b200",
    version="0.1.0",
    packages=find_packages(include=["vllm_neuron_b200", "vllm_neuron_b200.*"]),
    ext_modules=[
        CUDAExtension(
            name="vllm_neuron_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={
        "vllm.platform_plugins": ["b200 = vllm_neuron_b200:register"],
        "console_scripts": ["vllm-b200 = vllm_neuron_b200.entrypoints.cli:main"],
    },
)
