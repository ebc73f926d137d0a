"""Packaging for glm53_sparse_mla (B200 / sm_100a build).

`pip install .` (or `python setup.py build_py`) first compiles the two shared
objects in place with glm53_sparse_mla/build.py (nvcc for sm_100a, g++ for the
torch-op binding) and ships them as package data. The vLLM general-plugin
entry point keeps the reference's name and target (setup.py:48-56 there), so
an installed package registers the backend exactly as before; register() does
nothing unless VLLM_GLM53_CUDA_SPARSE_MLA is set.
"""

import os
import sys

from setuptools import setup
from setuptools.command.build_py import build_py

HERE = os.path.dirname(os.path.abspath(__file__))


class BuildWithKernels(build_py):
    def run(self):
        sys.path.insert(0, os.path.join(HERE, "glm53_sparse_mla"))
        import build as kernel_build  # glm53_sparse_mla/build.py, without importing the package

        kernel_build.build(verbose=True)
        super().run()


setup(
    name="glm53_sparse_mla",
    version="0.2.0",
    packages=["glm53_sparse_mla"],
    package_data={"glm53_sparse_mla": ["_C.so", "libglm53_sparse_mla.so"]},
    cmdclass={"build_py": BuildWithKernels},
    entry_points={
        "vllm.general_plugins": [
            "glm53_sparse_mla = glm53_sparse_mla.backend:register",
        ],
    },
)
