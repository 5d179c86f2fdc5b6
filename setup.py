"""Builds the two in-tree native modules of hawking_b200.

* ``hawking_b200._native``  host C++ (formats, CPU reference, engine, HTTP server); pybind11.
* ``hawking_b200._kernels`` sm_100a CUDA kernels plus their torch bindings.

Build in place (the .so files land next to the Python sources)::

    python setup.py build_ext --inplace

``HK_SKIP_CUDA=1`` builds only the host module.
"""
import glob
import os

import pybind11
from setuptools import Extension, setup

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("hawking_b200", "csrc")


def _sources(*patterns):
    out = []
    for p in patterns:
        out.extend(sorted(glob.glob(os.path.join(CSRC, p))))
    return out


CXX_FLAGS = ["-O3", "-std=c++17", "-pthread", "-fvisibility=hidden", "-Wno-unused-function"]
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

ext_modules = [
    Extension(
        "hawking_b200._native",
        sources=_sources("native/*.cpp", "bindings/native_module.cpp", "bindings/formats_bindings.cpp",
                         "bindings/engine_bindings.cpp", "bindings/serve_bindings.cpp"),
        # the CUDA toolkit's header-only NVTX (trace ranges) when present; no CUDA library is linked
        include_dirs=[pybind11.get_include(), os.path.join(ROOT, CSRC)] + (
            [os.path.join(CUDA_HOME, "include")] if os.path.isdir(os.path.join(CUDA_HOME, "include", "nvtx3")) else []),
        extra_compile_args=CXX_FLAGS,
        extra_link_args=["-pthread", "-ldl"],
        language="c++",
    )
]
cmdclass = {}

if os.environ.get("HK_SKIP_CUDA", "0") != "1":
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension

    NVCC_FLAGS = [
        "-O3", "-std=c++17", "-lineinfo",
        "-gencode", "arch=compute_100a,code=sm_100a",
        "--expt-relaxed-constexpr", "-Xptxas", "-v,-warn-spills" if os.environ.get("HK_PTXAS_V") else "-warn-spills",
        "-DNDEBUG",
    ]
    if os.environ.get("HK_BOUNDS", "0") == "1":
        NVCC_FLAGS.append("-DHK_BOUNDS=1")
    # tuning builds: extra preprocessor definitions, e.g. HK_NVCC_DEFINES="HK_MG_STAGES=4 HK_MG_TPC=1"
    NVCC_FLAGS += ["-D" + d for d in os.environ.get("HK_NVCC_DEFINES", "").split()]
    ext_modules.append(
        CUDAExtension(
            "hawking_b200._kernels",
            sources=_sources("kernels/*.cu", "bindings/kernels_module.cpp", "bindings/kernels_more.cpp",
                             "bindings/kernels_tp.cpp", "bindings/kernels_models.cpp",
                             "bindings/kernels_mg.cpp", "bindings/kernels_ds.cpp"),
            include_dirs=[os.path.join(ROOT, CSRC, "kernels")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            libraries=["cuda"],
        )
    )
    cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)

# Host-only builds (HK_SKIP_CUDA=1) compile without torch's BuildExtension, whose pybind11 ABI
# defines differ; separate object directories keep the two kinds of objects from being linked
# into one module.
_temp = "build/temp-host" if os.environ.get("HK_SKIP_CUDA", "0") == "1" else "build/temp-full"

setup(
    name="hawking_b200",
    version="0.1.0",
    packages=["hawking_b200"],
    ext_modules=ext_modules,
    cmdclass=cmdclass,
    options={"build_ext": {"build_temp": _temp}},
)
