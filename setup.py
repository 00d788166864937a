"""Build the harp_b200 CUDA extension in place (sm_100a):

    python setup.py build_ext --inplace

The extension library (harp_b200/_build/harp_b200_C.so) is compiled by
harp_b200._native with nvcc -gencode arch=compute_100a,code=sm_100a; this file
only wires that build into setuptools so `pip install -e .` works too.
"""
from setuptools import find_packages, setup
from setuptools.command.build_ext import build_ext


class HarpBuild(build_ext):
    def run(self):
        from harp_b200 import _native

        _native.build(verbose=True)


setup(
    name="harp_b200",
    version="0.1.0",
    description="Sequence-parallel DiT training on B200 (sm_100a): tcgen05 kernels, NVLink collectives",
    packages=find_packages(include=["harp_b200", "harp_b200.*"]),
    package_data={"harp_b200": ["csrc/*.cu", "csrc/*.cuh", "csrc/*.cpp", "csrc/*.h"]},
    python_requires=">=3.10",
    cmdclass={"build_ext": HarpBuild},
)
