"""Build the sm_100a kernel library in place: ``python setup.py build_ext --inplace``."""

from pathlib import Path

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "nano_megatron_b200" / "csrc"

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode=arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if False else "-Xptxas=-O3",
]


def extension() -> CUDAExtension:
    sources = sorted(str(p.relative_to(ROOT)) for p in CSRC.glob("*.cu")) + [
        str((CSRC / "bindings.cpp").relative_to(ROOT))
    ]
    return CUDAExtension(
        name="nano_megatron_b200._C",
        sources=sources,
        include_dirs=[str(CSRC)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        # no libcuda link: driver entry points are resolved through the runtime, so the
        # library also imports (for the build check) on hosts without a GPU driver
    )


def host_extension() -> CppExtension:
    """Host-only runtime (data loading); no CUDA dependency, so it imports on CPU hosts."""
    sources = sorted(str(p.relative_to(ROOT)) for p in (CSRC / "host").glob("*.cpp"))
    return CppExtension(
        name="nano_megatron_b200._native",
        sources=sources,
        extra_compile_args={"cxx": ["-O3", "-std=c++17", "-pthread"]},
        extra_link_args=["-pthread"],
    )


setup(
    name="nano-megatron-b200",
    version="0.1.0",
    packages=find_packages(include=["nano_megatron_b200", "nano_megatron_b200.*"]),
    ext_modules=[extension(), host_extension()],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={
        "console_scripts": [
            "nano-megatron-train=nano_megatron_b200.cli.train:main",
            "nano-megatron-export=nano_megatron_b200.cli.export:main",
            "nano-megatron-generate=nano_megatron_b200.cli.generate:main",
            "nano-megatron-tokenizer=nano_megatron_b200.cli.tokenizer:main",
            "nano-megatron-tinystories=nano_megatron_b200.cli.tinystories:main",
            "nano-megatron-validate-nccl=nano_megatron_b200.distributed.validate_nccl:main",
        ]
    },
)
