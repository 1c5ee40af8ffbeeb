"""Build of the in-tree sm_100a extension ``vllm_neuron_b200._C``.

``python setup.py build_ext --inplace`` compiles every CUDA source under ``csrc/`` for
sm_100a only and places the shared object next to the package, so it travels with the
source tree.
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

SM100 = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = SM100 + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]


def sources():
    cu = sorted(glob.glob(os.path.join("csrc", "**", "*.cu"), recursive=True))
    return ["csrc/bindings.cpp"] + cu


setup(
    name="vllm_neuron_b200",
    version="0.1.0",
    packages=find_packages(include=["vllm_neuron_b200", "vllm_neuron_b200.*"]),
    # vLLM discovers the B200 platform through this plugin group once the package is installed
    # (pip install -e .): `vllm serve` / vllm.LLM then run on this framework's worker.
    entry_points={"vllm.platform_plugins": ["b200 = vllm_neuron_b200.vllm_plugin:register"]},
    ext_modules=[
        CUDAExtension(
            name="vllm_neuron_b200._C",
            sources=sources(),
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
